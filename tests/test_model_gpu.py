"""Model-level parity on the GPU: the tiny CPU-runnable configuration (1 layer,
hidden 128, 2/2 heads, head_dim 64, float32, hot ring 8, blocks of 4) driven by
``rfsn_b200.model`` with the reference's weights, prompt and greedy decode,
against the logits, tokens and ring/page-table states the reference produced
(``tests/golden/tiny_model_golden.npz``). Attention runs on the CUDA kernels
(float32 cache -> CUDA-core kernel); prefill and 8 decode steps seal archived
blocks, so the segmented path is exercised."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from _util import GOLDEN
from test_model_cpu import tiny_config

pytestmark = pytest.mark.gpu
ATOL = 2e-3  # parity bar for logits (max-abs vs the float32 reference)
GUARD = 1e-4  # float32 end to end: observed ~1e-6


def _state(cache):
    lc = cache.layer(0)
    return [lc.hot_head_index, lc.hot_seq_len, lc.hot_start] + [
        x for m in lc.block_manager.iter_blocks(layer_id=0) for x in (m.logical_start, m.logical_end)
    ]


def test_tiny_model_matches_reference_logits_tokens_and_ring(tmp_path):
    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.model import RFSNModel

    g = np.load(GOLDEN / "tiny_model_golden.npz")
    cfg = tiny_config(tmp_path)
    model = RFSNModel(cfg, device="cuda")
    model.load_weights({k[2:]: g[k] for k in g.files if k.startswith("w/")})
    cache = RFSNCache(cfg, batch_size=1, device="cuda")
    ring = g["ring_states"]

    logits = model.prefill(g["prompt"], cache)
    err = float(np.abs(logits.cpu().numpy() - g["prefill_logits"]).max())
    assert err <= ATOL and err <= GUARD, err
    st = _state(cache)
    assert st == [int(x) for x in ring[0][:len(st)]] and all(x == -1 for x in ring[0][len(st):])

    token = torch.argmax(logits[:, -1, :], dim=-1).to(torch.int32)
    tokens = [int(token[0])]
    pos = 8
    for step in range(8):
        out = model.decode_step(token, cache, pos)
        err = float(np.abs(out.cpu().numpy() - g["decode_logits"][step]).max())
        assert err <= ATOL and err <= GUARD, (step, err)
        st = _state(cache)
        assert st == [int(x) for x in ring[step + 1][:len(st)]], (step, st)
        token = torch.argmax(out, dim=-1).to(torch.int32)
        tokens.append(int(token[0]))
        pos += 1
    assert tokens == [int(t) for t in g["tokens"]]


def test_generate_greedy_equals_stepwise(tmp_path):
    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.model import RFSNModel

    g = np.load(GOLDEN / "tiny_model_golden.npz")
    cfg = tiny_config(tmp_path, session_id="tiny-gen")
    model = RFSNModel(cfg, device="cuda")
    model.load_weights({k[2:]: g[k] for k in g.files if k.startswith("w/")})
    out = model.generate(g["prompt"], 9, cache=RFSNCache(cfg, batch_size=1, device="cuda"), temperature=0.0)
    assert [int(t[0]) for t in out] == [int(t) for t in g["tokens"]]


def test_bf16_model_prefill_chunks_and_decode_run_on_tensor_core_paths(tmp_path, monkeypatch):
    """A larger bf16 model (head_dim 128, GQA 4, 2 layers, hot ring 256, blocks of
    128): prefill chunks of 256/256/88 tokens go to the tcgen05 prefill kernel and
    decode steps to the split-KV decode kernel, over sealed archived blocks and a
    wrapped ring. Every attention call the model makes is checked against dense
    float32 attention over the full history of the same q/k/v (1e-4). A bf16
    network turns ~1e-6 differences into ulp-level noise downstream, so the logits
    are only checked against a dense re-computation to a few bf16 ulps."""
    import rfsn_b200.model as M
    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.config import RFSNConfig, RuntimeMode

    calls = []
    orig = M.attention_step

    def recording(q, k, v, layer_cache, start_pos):
        out = orig(q, k, v, layer_cache, start_pos)
        calls.append((layer_cache.layer_id, q.detach().clone(), k.detach().clone(), v.detach().clone(), start_pos,
                      out.detach().clone()))
        return out

    monkeypatch.setattr(M, "attention_step", recording)
    cfg = RFSNConfig(hidden_dim=1024, num_heads=8, num_kv_heads=2, head_dim=128, num_layers=2, vocab_size=256,
                     hot_capacity=256, block_size_seq=128, warm_capacity=4096, rope_base=10000.0, ffn_multiplier=2,
                     model_dtype="bfloat16", runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=str(tmp_path),
                     session_id="bf16")
    model = M.RFSNModel(cfg, device="cuda", seed=7)
    model.use_graphs = False  # every attention call goes through attention_step (recorded here)
    cache = RFSNCache(cfg, batch_size=1, device="cuda")
    dense = _DenseModel(model)
    prompt = torch.randint(0, 256, (1, 600), generator=torch.Generator().manual_seed(8))
    logits = model.prefill(prompt, cache)
    ref = torch.cat([dense(prompt[:, a:b]) for a, b in ((0, 256), (256, 512), (512, 600))], dim=1)
    _close_bf16(logits[0].float(), ref[0])
    tok = torch.argmax(logits[:, -1], dim=-1)
    for pos in range(600, 604):
        out = model.decode_step(tok, cache, pos)
        ref = dense(tok.reshape(1, 1).cpu())[:, -1]
        _close_bf16(out[0].float(), ref[0])
        tok = torch.argmax(out, dim=-1)
    assert len(calls) == 2 * (3 + 4)
    assert [c[1].shape[2] for c in calls[::2]] == [256, 256, 88, 1, 1, 1, 1]

    hist = {}
    for layer_id, q, k, v, start_pos, out in calls:
        kr = _rope(k, start_pos, cfg).to(torch.bfloat16).float()
        kh, vh = hist.get(layer_id, (None, None))
        kh = kr if kh is None else torch.cat([kh, kr], dim=2)
        vh = v.float() if vh is None else torch.cat([vh, v.float()], dim=2)
        hist[layer_id] = (kh, vh)
        qr = _rope(q, start_pos, cfg)
        G = cfg.num_heads // cfg.num_kv_heads
        s = qr @ kh.repeat_interleave(G, 1).transpose(-1, -2) / cfg.head_dim ** 0.5
        L, T = q.shape[2], kh.shape[2]
        qpos = torch.arange(start_pos, start_pos + L, device=q.device)[:, None]
        s = s.masked_fill(torch.arange(T, device=q.device)[None, :] > qpos, float("-inf"))
        want = torch.softmax(s, dim=-1) @ vh.repeat_interleave(G, 1)
        err = float((out - want).abs().max())
        assert err <= 1e-4, (layer_id, start_pos, L, err)


def _rope(t, start_pos, cfg):
    from rfsn_b200.layer import build_rope_tables

    D = cfg.head_dim
    cos, sin = build_rope_tables(D, cfg.rope_base, t.shape[2], start_pos, device=t.device)
    t = t.float()
    rot = torch.cat([-t[..., D // 2:], t[..., :D // 2]], dim=-1)
    return t * cos + rot * sin


def _close_bf16(got, ref):
    ulp = 2.0 ** -7 * float(ref.abs().max())  # bf16 spacing at the largest logit
    diff = (got - ref).abs()
    assert float(diff.max()) <= 4 * ulp, (float(diff.max()), ulp)
    assert float(diff.mean()) <= ulp / 2, (float(diff.mean()), ulp)


class _DenseModel:
    """The same network with plain dense attention (float32 softmax over all
    previous K/V, GQA by head mapping), fed the same chunks as the model so
    every projection runs with the same shapes (identical cuBLAS results); only
    the attention differs."""

    def __init__(self, model):
        self.m = model
        self.k = [None] * model.config.num_layers
        self.v = [None] * model.config.num_layers
        self.pos = 0

    def __call__(self, toks):
        import torch.nn.functional as F

        from rfsn_b200.layer import build_rope_tables
        from rfsn_b200.model import _layer_norm, _rms_norm

        m, cfg, p = self.m, self.m.config, self.m.params
        L = toks.shape[1]
        H, Hkv, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        cos, sin = build_rope_tables(D, cfg.rope_base, L, self.pos, device=m.device)

        def rope(t):
            t = t.float()
            rot = torch.cat([-t[..., D // 2:], t[..., :D // 2]], dim=-1)
            return t * cos + rot * sin

        x = F.embedding(toks.to(m.device).long(), p["embed_tokens.weight"])
        for i in range(cfg.num_layers):
            w = lambda n: p[f"layers.{i}.{n}"]  # noqa: E731
            xn = _rms_norm(x, w("attn_norm.weight"), cfg.norm_eps)
            q = rope(F.linear(xn, w("q_proj.weight")).reshape(1, L, H, D).transpose(1, 2))
            k = rope(F.linear(xn, w("k_proj.weight")).reshape(1, L, Hkv, D).transpose(1, 2)).to(m.dtype).float()
            v = F.linear(xn, w("v_proj.weight")).reshape(1, L, Hkv, D).transpose(1, 2).to(m.dtype).float()
            self.k[i] = k if self.k[i] is None else torch.cat([self.k[i], k], dim=2)
            self.v[i] = v if self.v[i] is None else torch.cat([self.v[i], v], dim=2)
            kk = self.k[i].repeat_interleave(H // Hkv, dim=1)
            vv = self.v[i].repeat_interleave(H // Hkv, dim=1)
            T = kk.shape[2]
            s = q @ kk.transpose(-1, -2) / D ** 0.5
            qpos = torch.arange(self.pos, self.pos + L, device=m.device)[:, None]
            s = s.masked_fill(torch.arange(T, device=m.device)[None, :] > qpos, float("-inf"))
            a = (torch.softmax(s, dim=-1) @ vv).transpose(1, 2).reshape(1, L, H * D).to(x.dtype)
            x = x + F.linear(a, w("o_proj.weight"))
            h = _rms_norm(x, w("ffn_norm.weight"), cfg.norm_eps)
            x = x + F.linear(F.silu(F.linear(h, w("gate_proj.weight"))) * F.linear(h, w("up_proj.weight")),
                             w("down_proj.weight"))
        x = _layer_norm(x, p["norm.weight"], p["norm.bias"], cfg.norm_eps)
        self.pos += L
        return (x @ p["embed_tokens.weight"].T).float()


def test_decode_graph_matches_op_by_op_decode(tmp_path):
    """The captured whole-model decode step (device step state, re-captured after
    every seal) against op-by-op decoding of the same model and tokens: equal
    cache states; logits equal up to bf16 noise (the graph's decode kernel plans
    its splits for the largest hot window, so float32 sums run in another order)."""
    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.config import RFSNConfig, RuntimeMode
    from rfsn_b200.model import RFSNModel

    def make(use_graphs, sub):
        cfg = RFSNConfig(hidden_dim=1024, num_heads=8, num_kv_heads=2, head_dim=128, num_layers=3, vocab_size=512,
                         hot_capacity=128, block_size_seq=64, warm_capacity=4096, rope_base=10000.0,
                         ffn_multiplier=2, model_dtype="bfloat16", runtime_mode=RuntimeMode.ARCHIVED,
                         disk_cache_dir=str(tmp_path / sub), session_id=sub)
        m = RFSNModel(cfg, device="cuda", seed=11)
        m.use_graphs = use_graphs
        return m, RFSNCache(cfg, batch_size=1, device="cuda")

    eager, c_e = make(False, "eager")
    graphed, c_g = make(True, "graph")
    prompt = torch.randint(0, 512, (1, 100), generator=torch.Generator().manual_seed(12))
    le, lg = eager.prefill(prompt, c_e), graphed.prefill(prompt, c_g)
    tok = torch.argmax(le[:, -1], dim=-1).to(torch.int32)
    for pos in range(100, 100 + 150):  # seals every 64 tokens once the 128-token ring is full
        oe = eager.decode_step(tok, c_e, pos)
        og = graphed.decode_step(tok, c_g, pos)
        _close_bf16(og[0].float(), oe[0].float())
        for a, b in zip(c_e.layers, c_g.layers):
            assert (a.hot_head_index, a.hot_seq_len, a.hot_start) == (b.hot_head_index, b.hot_seq_len, b.hot_start)
            assert [(m.logical_start, m.logical_end) for m in a.block_manager.iter_blocks(layer_id=a.layer_id)] == \
                   [(m.logical_start, m.logical_end) for m in b.block_manager.iter_blocks(layer_id=b.layer_id)]
        tok = torch.argmax(oe, dim=-1).to(torch.int32)  # both models are fed the same tokens
    g = graphed._graph
    assert g is not None and g.replays > 100 and 2 <= g.captures <= 8, (g.replays, g.captures)
    graphed._graph.workspace.check()


def test_decode_graph_falls_back_when_blocks_are_cold(tmp_path):
    """A warm capacity below the archived context leaves cold blocks: the step
    runs op by op (reloads included) and matches the op-by-op model exactly."""
    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.config import RFSNConfig, RuntimeMode
    from rfsn_b200.model import RFSNModel

    def make(use_graphs, sub):
        cfg = RFSNConfig(hidden_dim=512, num_heads=4, num_kv_heads=1, head_dim=128, num_layers=1, vocab_size=256,
                         hot_capacity=64, block_size_seq=32, warm_capacity=64, cold_capacity=4096, rope_base=10000.0,
                         ffn_multiplier=2, model_dtype="bfloat16", runtime_mode=RuntimeMode.ARCHIVED,
                         disk_cache_dir=str(tmp_path / sub), session_id=sub)
        m = RFSNModel(cfg, device="cuda", seed=13)
        m.use_graphs = use_graphs
        return m, RFSNCache(cfg, batch_size=1, device="cuda")

    eager, c_e = make(False, "e")
    graphed, c_g = make(True, "g")
    for c in (c_e, c_g):  # prefetch loads on the caller's thread: one residency schedule for both models
        c.layer(0).residency_manager.inline_loads = True
    prompt = torch.randint(0, 256, (1, 200), generator=torch.Generator().manual_seed(14))
    le = eager.prefill(prompt, c_e)
    graphed.prefill(prompt, c_g)
    tok = torch.argmax(le[:, -1], dim=-1).to(torch.int32)
    for pos in range(200, 210):
        c_e.layer(0).residency_manager.wait_for_prefetches(c_e.layer(0), timeout=30.0)
        c_g.layer(0).residency_manager.wait_for_prefetches(c_g.layer(0), timeout=30.0)
        oe = eager.decode_step(tok, c_e, pos)
        og = graphed.decode_step(tok, c_g, pos)
        assert torch.equal(oe, og)
        tok = torch.argmax(oe, dim=-1).to(torch.int32)
    assert c_g.layer(0).residency_manager.get_metrics() == c_e.layer(0).residency_manager.get_metrics()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fused_rms_norm_and_swiglu_match_the_elementwise_formulas(dtype):
    """rfsn_rms_norm / rfsn_silu_mul against the reference's elementwise
    formulas (layer.py:54-64, :94-95) evaluated in torch: equal up to one
    rounding of the storage type (different summation order of the mean)."""
    from rfsn_b200.model import _add_rms_norm, _rms_norm, _silu_mul

    gen = torch.Generator(device="cuda").manual_seed(11)
    for rows, n in ((1, 4096), (7, 128), (3, 1000)):
        x = (torch.randn((rows, n), generator=gen, device="cuda") * 3).to(dtype)
        w = (torch.rand((n,), generator=gen, device="cuda") + 0.5).to(dtype)
        xf = x.float()
        want = (w.float() * (xf / torch.sqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + 1e-5))).to(dtype)
        got = _rms_norm(x, w, 1e-5)
        ulp = {torch.float32: 2e-6, torch.bfloat16: 8e-3, torch.float16: 1e-3}[dtype]
        assert torch.allclose(got.float(), want.float(), rtol=ulp, atol=ulp), (rows, n)
        if n % 8 == 0:  # residual add fused in (16-byte rows)
            r = torch.randn((rows, n), generator=gen, device="cuda").to(dtype)
            s_want = r + x
            sf = s_want.float()
            want = (w.float() * (sf / torch.sqrt(torch.mean(sf * sf, dim=-1, keepdim=True) + 1e-5))).to(dtype)
            s_got, got = _add_rms_norm(x, r, w, 1e-5)
            assert torch.equal(s_got, s_want), (rows, n)
            assert torch.allclose(got.float(), want.float(), rtol=ulp, atol=ulp), (rows, n)
        gu = (torch.randn((rows, 2 * n), generator=gen, device="cuda") * 4).to(dtype)
        want = F.silu(gu[:, :n]) * gu[:, n:]
        got = _silu_mul(gu)
        assert torch.allclose(got.float(), want.float(), rtol=ulp, atol=ulp), (rows, n)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,n,k", [(1, 4096, 4096), (1, 6144, 4096), (1, 1000, 14336), (3, 257, 512), (4, 96, 128)])
def test_decode_gemv_matches_float32_product(dtype, rows, n, k):
    """rfsn_gemv (the model's decode projections) against the float32 product
    rounded once: within one rounding of the storage type."""
    from rfsn_b200.model import _linear

    gen = torch.Generator(device="cuda").manual_seed(rows * 7 + n)
    w = (torch.randn((n, k), generator=gen, device="cuda") * 0.05).to(dtype)
    x = torch.randn((rows, k), generator=gen, device="cuda").to(dtype)
    want = (x.double() @ w.double().T).float()
    got = _linear(x, w).float()
    tol = {torch.float32: 1e-4, torch.bfloat16: 1.6e-2, torch.float16: 2e-3}[dtype]
    assert torch.allclose(got, want, rtol=tol, atol=tol * float(want.abs().max())), float((got - want).abs().max())


def test_standalone_layer_matches_the_model_layer(tmp_path):
    """RFSNLayerMLX(config, 0) with the model's layer-0 weights, called with the
    reference's positional signature (x, cache, rope_tables, start_pos), gives
    the model layer's output and cache state."""
    from rfsn_b200 import RFSNCache, RFSNLayerMLX, RFSNModel

    cfg = tiny_config(tmp_path / "a")
    model = RFSNModel(cfg, device="cuda", seed=3)
    layer = RFSNLayerMLX(cfg, 0, device="cuda")
    for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "attn_norm",
                 "ffn_norm"):
        getattr(layer, name).weight.copy_(getattr(model.layers[0], name).weight)
    c1 = RFSNCache(cfg, batch_size=1, device="cuda")
    c2 = RFSNCache(tiny_config(tmp_path / "b"), batch_size=1, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(5)
    pos = 0
    for L in (6, 1, 1, 5):  # prefill-like chunks and decode steps across seals of the 8-token ring
        x = torch.randn((1, L, cfg.hidden_dim), generator=gen, device="cuda")
        a = model.layers[0](x, c1.layer(0), start_pos=pos)
        b = layer(x, c2.layer(0), None, pos)
        assert torch.equal(a, b)
        pos += L
    l1, l2 = c1.layer(0), c2.layer(0)
    assert (l1.hot_head_index, l1.hot_seq_len, l1.hot_start) == (l2.hot_head_index, l2.hot_seq_len, l2.hot_start)


def _golden_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("name", ["cfg4_slice", "cfg5_slice"])
def test_model_slice_at_8b_and_7b_head_geometry_matches_reference(tmp_path, name):
    """Two float32 layers at the head geometry of the Llama-3-8B- and
    Mistral-7B-shaped configurations (head_dim 128, 8 q / 2 kv heads = GQA 4,
    RoPE theta 5e5 / 1e6, hidden 1024, FFN 3584) with a small ring, blocks and
    warm capacity: the chunked prompt seals blocks, half of them go cold, and
    every decode step reloads them (the reference's policy) while prefetching;
    prefetch loads run when scheduled on both sides, so the residency decisions
    follow one deterministic schedule.
    Logits, greedy tokens, layer 0's ring / page-table / residency states after
    every step and both layers' residency counters equal the reference's
    (tests/golden/model_slices_golden.npz, model.py:106-189 and
    residency.py:85-145 run over the torch shim)."""
    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.config import RFSNConfig, RuntimeMode
    from rfsn_b200.model import RFSNModel

    mg = _golden_module()
    g = np.load(GOLDEN / "model_slices_golden.npz")
    _, seed, over, n_prompt, n_decode = next(c for c in mg.MODEL_SLICES if c[0] == name)
    cfg = RFSNConfig(**mg.SLICE_DIMS, **over, runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=str(tmp_path),
                     session_id=name.replace("_", "-"))
    model = RFSNModel(cfg, device="cuda")
    model.load_weights(mg.slice_weights(model.parameter_shapes(), seed))
    cache = RFSNCache(cfg, batch_size=1, device="cuda")
    for i in range(cfg.num_layers):  # prefetches complete when scheduled, as in the fixture
        cache.layer(i).residency_manager.inline_loads = True

    def state():
        lc = cache.layer(0)
        return [lc.hot_head_index, lc.hot_seq_len, lc.hot_start] + [
            x for m in lc.block_manager.iter_blocks(layer_id=0)
            for x in (m.logical_start, m.logical_end, 1 if m.residency.value == "warm_ram" else 0)]

    ring = g[f"{name}/ring_states"]

    def check_state(i):
        st = state()
        assert st == [int(x) for x in ring[i][:len(st)]] and all(x == -1 for x in ring[i][len(st):]), (i, st)

    logits = model.prefill(g[f"{name}/prompt"], cache)
    err = float(np.abs(logits.cpu().numpy() - g[f"{name}/prefill_logits"]).max())
    assert err <= ATOL and err <= GUARD, err
    check_state(0)
    token = torch.argmax(logits[:, -1, :], dim=-1).to(torch.int32)
    tokens = [int(token[0])]
    pos = n_prompt
    for step in range(n_decode):
        out = model.decode_step(token, cache, pos)
        err = float(np.abs(out.cpu().numpy() - g[f"{name}/decode_logits"][step]).max())
        assert err <= ATOL and err <= GUARD, (step, err)
        check_state(step + 1)
        token = torch.argmax(out, dim=-1).to(torch.int32)
        tokens.append(int(token[0]))
        pos += 1
    assert tokens == [int(t) for t in g[f"{name}/tokens"]]
    for i in range(cfg.num_layers):
        m = cache.layer(i).residency_manager.get_metrics()
        assert [m[k] for k in sorted(m)] == [int(x) for x in g[f"{name}/residency_metrics"][i]], (i, m)
