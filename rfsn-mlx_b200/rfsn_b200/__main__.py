"""Command line: ``python -m rfsn_b200 bench [model flags] [bench flags]``.

Mirrors the ``bench`` subcommand of the reference launcher
(launcher.py:237-268, flags at :316-345 and :370-378): builds a randomly
initialised model from the flags, prints the model line, then the prefill and
decode ``BenchResult`` lines.
"""

from __future__ import annotations

import argparse
import sys
from typing import List, Optional


def _add_model_args(p: argparse.ArgumentParser) -> None:
    p.add_argument("--hidden-dim", type=int, default=512)
    p.add_argument("--num-heads", type=int, default=8)
    p.add_argument("--num-kv-heads", type=int, default=0, help="KV heads for GQA (0 = same as num-heads)")
    p.add_argument("--head-dim", type=int, default=64)
    p.add_argument("--num-layers", type=int, default=4)
    p.add_argument("--vocab-size", type=int, default=50000)
    p.add_argument("--rope-base", type=float, default=10000.0)
    p.add_argument("--ffn-dim", type=int, default=0)
    p.add_argument("--hot-capacity", type=int, default=512)
    p.add_argument("--warm-capacity", type=int, default=2048)
    p.add_argument("--cold-capacity", type=int, default=8192)
    p.add_argument("--block-size-seq", type=int, default=64)
    p.add_argument("--runtime-mode", type=str, default="archived", choices=["exact", "archived"],
                   help="'archived' spills exact sealed prefixes to archived blocks; 'exact' is hot-window only")
    p.add_argument("--disk-cache-dir", type=str, default="./rfsn_disk_cache")
    p.add_argument("--session-id", type=str, default="",
                   help="Explicit cache session identifier; auto-generated otherwise.")
    p.add_argument("--model-dtype", type=str, default="bfloat16", choices=["float16", "bfloat16", "float32"])


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m rfsn_b200", description="RFSN B200 exact segmented attention")
    sub = ap.add_subparsers(dest="command", required=True)
    bnc = sub.add_parser("bench", help="Run prefill and decode benchmarks")
    _add_model_args(bnc)
    bnc.add_argument("--prompt-len", type=int, default=256)
    bnc.add_argument("--decode-steps", type=int, default=100)
    bnc.add_argument("--warmup", type=int, default=2)
    bnc.add_argument("--repeats", type=int, default=5)
    bnc.add_argument("--seed-prompt-len", type=int, default=8)
    bnc.add_argument("--archive-seed-steps", type=int, default=0)
    bnc.add_argument("--seed", type=int, default=0, help="random-init seed of the model weights")
    return ap


def config_from_args(args: argparse.Namespace):
    from .config import RFSNConfig

    return RFSNConfig(
        hidden_dim=args.hidden_dim, num_heads=args.num_heads, num_kv_heads=args.num_kv_heads,
        head_dim=args.head_dim, num_layers=args.num_layers, vocab_size=args.vocab_size, rope_base=args.rope_base,
        ffn_dim=args.ffn_dim, hot_capacity=args.hot_capacity, warm_capacity=args.warm_capacity,
        cold_capacity=args.cold_capacity, block_size_seq=args.block_size_seq, runtime_mode=args.runtime_mode,
        disk_cache_dir=args.disk_cache_dir, session_id=args.session_id, model_dtype=args.model_dtype,
    )


def cmd_bench(args: argparse.Namespace) -> None:
    from .bench import bench_decode, bench_prefill
    from .cache import RFSNCache
    from .model import RFSNModel

    config = config_from_args(args)
    model = RFSNModel(config, seed=args.seed)
    cache = RFSNCache(config, batch_size=1, device=model.device)
    print(
        f"[bench] Model: {config.num_layers}L x {config.hidden_dim}d, "
        f"{config.num_heads}H/{config.num_kv_heads}KVH, "
        f"dtype={config.model_dtype}, runtime_mode={config.runtime_mode.value}, session_id={cache.session_id}"
    )
    print(bench_prefill(model, cache, prompt_len=args.prompt_len, warmup=args.warmup, repeats=args.repeats))
    print(bench_decode(model, cache, steps=args.decode_steps, warmup=args.warmup, repeats=args.repeats,
                       seed_prompt_len=args.seed_prompt_len, archive_seed_steps=args.archive_seed_steps))


def main(argv: Optional[List[str]] = None) -> int:
    args = build_parser().parse_args(argv)
    if args.command == "bench":
        cmd_bench(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
