"""Model driver (drop-in for ``rfsn_v10_5.model.RFSNMLX``, model.py:43-336).

The transformer around the attention path: token embedding, per layer
RMSNorm -> q/k/v projections -> attention step -> o_proj + residual ->
RMSNorm -> SwiGLU FFN + residual (layer.py:53-167), final LayerNorm and a
weight-tied LM head (model.py:56-69). Prefill runs in chunks of
``min(hot_capacity, L)`` tokens at ``start_pos = cache.layer(0).hot_end``
(model.py:133-165); decode validates ``pos == hot_end`` (model.py:89-104).

The attention step of every layer is ``layer.attention_step``: RoPE fused
with the ring append, the seal rule, the decode prefetch hook and exact
attention over archived blocks + hot window on the CUDA kernels. The dense
projections, norms and FFN are plain torch operations on the same device.

Parameter names follow the reference's ``tree_flatten(model.parameters())``
(``embed_tokens.weight``, ``layers.{i}.q_proj.weight``, ...,
``layers.{i}.attn_norm.weight``, ``norm.weight``, ``norm.bias``) so weights
load unchanged. Activations stay in the model dtype (the float32 attention
output is cast back before ``o_proj``); for a float32 model this is the
reference's dtype flow.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Mapping, Optional, Tuple, Union

import numpy as np
import torch
import torch.nn.functional as F

from . import _native as native
from .cache import RFSNCache, _as, paged_attention
from .config import RFSNConfig, RuntimeMode, resolve_dtype
from .layer import attention_step, attention_step_tables, capture_graph

ArrayLike = Union[np.ndarray, torch.Tensor]


def _dense_device_check(x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise native.NativeUnavailable("the model's layers run on a CUDA device (no CPU path)")


def _rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """layer.py:54-64: weight * x / sqrt(mean(x^2) + eps), computed in float32
    and rounded once (one fused kernel, ``rfsn_rms_norm``)."""
    _dense_device_check(x)
    xc = x.contiguous()
    out = torch.empty_like(xc)
    n = int(xc.shape[-1])
    native.check(native.lib().rfsn_rms_norm(xc.data_ptr(), None, weight.data_ptr(), None, out.data_ptr(),
                                            xc.numel() // n, n, native.dtype_code(xc.dtype), float(eps),
                                            native.stream_ptr()), "rfsn_rms_norm")
    return out


def _add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                  eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(s, norm(s)) with s = residual + x in the storage type (the layer's
    residual add and the following RMSNorm as one kernel)."""
    _dense_device_check(x)
    xc, rc = x.contiguous(), residual.contiguous()
    s, out = torch.empty_like(xc), torch.empty_like(xc)
    n = int(xc.shape[-1])
    native.check(native.lib().rfsn_rms_norm(xc.data_ptr(), rc.data_ptr(), weight.data_ptr(), s.data_ptr(),
                                            out.data_ptr(), xc.numel() // n, n, native.dtype_code(xc.dtype),
                                            float(eps), native.stream_ptr()), "rfsn_rms_norm")
    return s, out


_GEMV_MAX_ROWS = 4


def _linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x @ w^T. Decode-sized inputs (<= 4 rows, 16-byte weight rows) run on this
    library's GEMV (``rfsn_gemv``: weights streamed once with 16-byte loads,
    float32 accumulation); larger ones on cuBLAS (``F.linear``)."""
    K = int(x.shape[-1])
    rows = x.numel() // K
    vec = 16 // x.element_size()
    if (x.is_cuda and rows <= _GEMV_MAX_ROWS and x.dtype == w.dtype and w.is_contiguous() and K % vec == 0
            and w.data_ptr() % 16 == 0 and rows * K * 4 <= 200 * 1024):
        xc = x.contiguous()
        y = torch.empty(tuple(x.shape[:-1]) + (int(w.shape[0]),), dtype=x.dtype, device=x.device)
        native.check(native.lib().rfsn_gemv(w.data_ptr(), xc.data_ptr(), y.data_ptr(), int(w.shape[0]), K, rows,
                                            native.dtype_code(x.dtype), native.stream_ptr()), "rfsn_gemv")
        return y
    return F.linear(x, w)


def _silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """layer.py:94-95 on a fused gate|up projection [..., 2F]: silu(gate) * up
    (one kernel, ``rfsn_silu_mul``)."""
    _dense_device_check(gate_up)
    gu = gate_up.contiguous()
    n = int(gu.shape[-1]) // 2
    out = torch.empty(tuple(gu.shape[:-1]) + (n,), dtype=gu.dtype, device=gu.device)
    native.check(native.lib().rfsn_silu_mul(gu.data_ptr(), out.data_ptr(), gu.numel() // (2 * n), n,
                                            native.dtype_code(gu.dtype), native.stream_ptr()), "rfsn_silu_mul")
    return out


def _layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    """model.py:65 (nn.LayerNorm): (x - mean) / sqrt(var + eps) * weight + bias."""
    return F.layer_norm(x.float(), (x.shape[-1],), weight.float(), bias.float(), eps).to(x.dtype)


def _layer_param_shapes(config: RFSNConfig, layer_idx: int) -> Dict[str, Tuple[int, ...]]:
    Hd, H, Hkv, D, Fd = config.hidden_dim, config.num_heads, config.num_kv_heads, config.head_dim, config.ffn_dim
    pre = f"layers.{layer_idx}."
    return {
        pre + "q_proj.weight": (H * D, Hd), pre + "k_proj.weight": (Hkv * D, Hd),
        pre + "v_proj.weight": (Hkv * D, Hd), pre + "o_proj.weight": (Hd, H * D),
        pre + "gate_proj.weight": (Fd, Hd), pre + "up_proj.weight": (Fd, Hd),
        pre + "down_proj.weight": (Hd, Fd),
        pre + "attn_norm.weight": (Hd,), pre + "ffn_norm.weight": (Hd,),
    }


def _fused_layer_storage(config: RFSNConfig, layer_idx: int, params: Dict[str, torch.Tensor], device: torch.device,
                         dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """Allocate one layer's q|k|v and gate|up matrices and register the named
    projection parameters as row views of them."""
    H, Hkv, D, Hd, Fd = config.num_heads, config.num_kv_heads, config.head_dim, config.hidden_dim, config.ffn_dim
    pre = f"layers.{layer_idx}."
    w_qkv = torch.empty(((H + 2 * Hkv) * D, Hd), device=device, dtype=dtype)
    w_gu = torch.empty((2 * Fd, Hd), device=device, dtype=dtype)
    params[pre + "q_proj.weight"] = w_qkv[:H * D]
    params[pre + "k_proj.weight"] = w_qkv[H * D:(H + Hkv) * D]
    params[pre + "v_proj.weight"] = w_qkv[(H + Hkv) * D:]
    params[pre + "gate_proj.weight"] = w_gu[:Fd]
    params[pre + "up_proj.weight"] = w_gu[Fd:]
    return w_qkv, w_gu


def _init_params(shapes: Mapping[str, Tuple[int, ...]], params: Dict[str, torch.Tensor], device: torch.device,
                 dtype: torch.dtype, gen: torch.Generator) -> None:
    """Random init normal(0, 0.02) in ``shapes`` order (norms: ones / zeros),
    written into existing views or stored as new tensors."""
    for name, shape in shapes.items():
        if name.endswith("norm.weight"):
            t = torch.ones(shape, device=device, dtype=dtype)
        elif name == "norm.bias":
            t = torch.zeros(shape, device=device, dtype=dtype)
        else:
            t = torch.empty(shape, device=device, dtype=torch.float32).normal_(0.0, 0.02, generator=gen).to(dtype)
        if name in params:
            params[name].copy_(t)
        else:
            params[name] = t


class _Weight:
    """A projection of the layer with the reference module's ``.weight``
    attribute (a view of the layer's parameter)."""

    __slots__ = ("weight",)

    def __init__(self, weight: torch.Tensor) -> None:
        self.weight = weight


class _ModelRopeTables:
    """The float32 RoPE tables the model builds for its layers (model.py:120,
    build_rope_tables with its default float32 dtype). The fused RoPE/append
    kernel computes exactly those rotations, so the tables are not built."""

    def __repr__(self) -> str:
        return "MODEL_ROPE_TABLES"


MODEL_ROPE_TABLES = _ModelRopeTables()


class RFSNLayerNorm:
    """layer.py:53-64 RMS norm (no bias): ``weight`` (ones unless given) and
    ``eps``; ``norm(x)`` is weight * x / sqrt(mean(x^2) + eps) computed in float32
    by the fused kernel and returned in x's dtype (the weight is read in x's
    dtype)."""

    def __init__(self, dim: int, eps: float = 1e-5, *, weight: Optional[torch.Tensor] = None,
                 device: Optional[Union[str, torch.device]] = None, dtype: torch.dtype = torch.float32) -> None:
        if weight is None:
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            weight = torch.ones((dim,), device=dev, dtype=dtype)
        if tuple(weight.shape) != (dim,):
            raise ValueError(f"RMS norm weight must have shape ({dim},), got {tuple(weight.shape)}")
        self.weight = weight
        self.eps = eps

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight if self.weight.dtype == x.dtype else self.weight.to(x.dtype)
        return _rms_norm(x, w, self.eps)


class RFSNLayer:
    """One transformer layer (layer.py:67-167) with the attention step on the CUDA path.

    ``RFSNLayer(config, layer_idx)`` (the reference's ``RFSNLayerMLX``
    constructor) builds a standalone layer with its own parameters, drawn
    normal(0, 0.02) (norms ones) on ``device`` (default: the current CUDA
    device); the model passes its parameter dict and fused matrices instead.
    The reference's ``q_proj`` ... ``down_proj``, ``attn_norm`` and
    ``ffn_norm`` attributes expose ``.weight`` views of the parameters."""

    def __init__(self, config: RFSNConfig, layer_idx: int, params: Optional[Dict[str, torch.Tensor]] = None,
                 w_qkv: Optional[torch.Tensor] = None, w_gate_up: Optional[torch.Tensor] = None, *,
                 device: Optional[Union[str, torch.device]] = None, seed: Optional[int] = None) -> None:
        self.config = config
        self.layer_idx = layer_idx
        if params is None:
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            dtype = resolve_dtype(config.model_dtype)
            params = {}
            w_qkv, w_gate_up = _fused_layer_storage(config, layer_idx, params, dev, dtype)
            gen = torch.Generator(device=dev)
            gen.manual_seed(layer_idx if seed is None else seed)
            _init_params(_layer_param_shapes(config, layer_idx), params, dev, dtype, gen)
        elif w_qkv is None or w_gate_up is None:
            raise ValueError("a layer built from a parameter dict needs its fused q|k|v and gate|up matrices")
        self.p = params  # the model's (or the layer's own) parameter dict
        # q|k|v and gate|up projections stored as one matrix each (the named
        # parameters are views of their rows): one GEMV instead of three / two
        self.w_qkv = w_qkv
        self.w_gate_up = w_gate_up
        for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
            setattr(self, name, _Weight(self._w(f"{name}.weight")))
        self.attn_norm = RFSNLayerNorm(config.hidden_dim, config.norm_eps, weight=self._w("attn_norm.weight"))
        self.ffn_norm = RFSNLayerNorm(config.hidden_dim, config.norm_eps, weight=self._w("ffn_norm.weight"))

    def _w(self, name: str) -> torch.Tensor:
        return self.p[f"layers.{self.layer_idx}.{name}"]

    def __call__(self, x: torch.Tensor, cache, rope_tables=None, start_pos: int = 0, attn=None) -> torch.Tensor:
        """layer.py:97-167. RoPE as the reference's layer applies it:
        ``rope_tables=MODEL_ROPE_TABLES`` (what ``RFSNModel`` passes: the float32
        tables of model.py:120) rotates in float32 inside the fused RoPE/append
        kernel; a (cos, sin) pair of tensors is used as given; None builds the
        tables in the model dtype (layer.py:118-126), with each product and sum
        rounded to the promoted dtype (for a float32 model that is the fused
        float32 path). ``attn(q, k, v)`` replaces the attention step (used by
        the captured decode graph)."""
        layer_cache = cache
        cfg = self.config
        B, L, _ = x.shape
        H, Hkv, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        residual = x
        xn = _rms_norm(x, self._w("attn_norm.weight"), cfg.norm_eps)
        qkv = _linear(xn, self.w_qkv)
        q = qkv[..., :H * D].reshape(B, L, H, D).transpose(1, 2)
        k = qkv[..., H * D:(H + Hkv) * D].reshape(B, L, Hkv, D).transpose(1, 2)
        v = qkv[..., (H + Hkv) * D:].reshape(B, L, Hkv, D).transpose(1, 2)
        if attn is not None:
            a = attn(q, k, v)  # float32 [B, H, L, D]
        elif rope_tables is MODEL_ROPE_TABLES or (rope_tables is None and layer_cache.dtype == torch.float32):
            a = attention_step(q, k, v, layer_cache, start_pos)
        else:
            a = attention_step_tables(q, k, v, layer_cache, start_pos, rope_tables)
        attn = a.transpose(1, 2).reshape(B, L, H * D).to(x.dtype)
        x, h = _add_rms_norm(_linear(attn, self._w("o_proj.weight")), residual, self._w("ffn_norm.weight"),
                             cfg.norm_eps)
        ffn = _linear(_silu_mul(_linear(h, self.w_gate_up)), self._w("down_proj.weight"))
        return x + ffn


class RFSNModel:
    """Full RFSN transformer (model.py:43-336)."""

    def __init__(self, config: RFSNConfig, *, device: Optional[Union[str, torch.device]] = None,
                 seed: Optional[int] = None) -> None:
        self.config = config
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = resolve_dtype(config.model_dtype)
        self.params: Dict[str, torch.Tensor] = {}
        # random init normal(0, 0.02) drawn on the model's device (an 8B-parameter
        # model initialises in seconds); norms start at ones / zeros
        gen = torch.Generator(device=self.device)
        gen.manual_seed(0 if seed is None else seed)
        # the fused matrices own the q/k/v and gate/up rows
        fused = [_fused_layer_storage(config, i, self.params, self.device, self.dtype) for i in range(config.num_layers)]
        _init_params(self.parameter_shapes(), self.params, self.device, self.dtype, gen)
        self.layers = [RFSNLayer(config, i, self.params, *fused[i]) for i in range(config.num_layers)]
        self.use_graphs = True
        self._graph: Optional["_DecodeGraph"] = None

    # ------------------------------------------------------------------ parameters
    def parameter_shapes(self) -> Dict[str, Tuple[int, ...]]:
        cfg = self.config
        Hd = cfg.hidden_dim
        shapes = {"embed_tokens.weight": (cfg.vocab_size, Hd), "norm.weight": (Hd,), "norm.bias": (Hd,)}
        for i in range(cfg.num_layers):
            shapes.update(_layer_param_shapes(cfg, i))
        return shapes

    def parameters(self) -> Dict[str, torch.Tensor]:
        return dict(self.params)

    def load_weights(self, weights: Union[Mapping[str, ArrayLike], Iterable[Tuple[str, ArrayLike]]],
                     strict: bool = False) -> "RFSNModel":
        """Load named weights (reference parameter names); ``strict`` requires every parameter."""
        items = weights.items() if isinstance(weights, Mapping) else list(weights)
        shapes = self.parameter_shapes()
        seen = set()
        for name, value in items:
            if name not in shapes:
                raise ValueError(f"Received parameter not in model: {name}")
            t = torch.as_tensor(np.asarray(value)) if isinstance(value, np.ndarray) else torch.as_tensor(value)
            if tuple(t.shape) != shapes[name]:
                raise ValueError(f"Expected shape {shapes[name]} for parameter {name} but received shape {tuple(t.shape)}")
            self.params[name].copy_(t.to(device=self.device, dtype=self.dtype))
            seen.add(name)
        if strict:
            missing = sorted(set(shapes) - seen)
            if missing:
                raise ValueError(f"Missing parameters: {missing}")
        return self

    # ------------------------------------------------------------------ driver
    def _lm_head(self, x: torch.Tensor) -> torch.Tensor:
        """model.py:67-69: weight-tied head x @ E^T."""
        return x @ self.params["embed_tokens.weight"].T

    def _context_end(self, cache: RFSNCache) -> int:
        return cache.layer(0).hot_end

    def _validate_prefill_bounds(self, cache: RFSNCache, incoming_tokens: int) -> int:
        """model.py:74-87 (same messages)."""
        context_end = self._context_end(cache)
        projected = context_end + incoming_tokens
        cfg = self.config
        if cfg.max_position_embeddings > 0 and projected > cfg.max_position_embeddings:
            raise ValueError(
                f"Prompt would exceed max_position_embeddings={cfg.max_position_embeddings} "
                f"(requested {projected} tokens total)"
            )
        if cfg.runtime_mode == RuntimeMode.EXACT and projected > cfg.hot_capacity:
            raise RuntimeError(
                "runtime_mode='exact' is hot-window only; the prompt would exceed "
                f"hot_capacity={cfg.hot_capacity}"
            )
        return context_end

    def _validate_decode_bounds(self, cache: RFSNCache, pos: int) -> None:
        """model.py:89-104 (same messages)."""
        context_end = self._context_end(cache)
        if pos != context_end:
            raise ValueError(f"decode_step expected pos={context_end} from cache state, got pos={pos}")
        projected = pos + 1
        cfg = self.config
        if cfg.max_position_embeddings > 0 and projected > cfg.max_position_embeddings:
            raise ValueError(f"Decode would exceed max_position_embeddings={cfg.max_position_embeddings}")
        if cfg.runtime_mode == RuntimeMode.EXACT and projected > cfg.hot_capacity:
            raise RuntimeError(
                "runtime_mode='exact' is hot-window only; the decode step would exceed "
                f"hot_capacity={cfg.hot_capacity}"
            )

    def _embed(self, tokens: torch.Tensor) -> torch.Tensor:
        return F.embedding(tokens.to(device=self.device, dtype=torch.long), self.params["embed_tokens.weight"])

    def _forward(self, x: torch.Tensor, cache: RFSNCache, start_pos: int) -> torch.Tensor:
        """model.py:106-131."""
        for i, layer in enumerate(self.layers):
            x = layer(x, cache.layer(i), rope_tables=MODEL_ROPE_TABLES, start_pos=start_pos)
        x = _layer_norm(x, self.params["norm.weight"], self.params["norm.bias"], self.config.norm_eps)
        return self._lm_head(x)

    def prefill(self, tokens: ArrayLike, cache: RFSNCache) -> torch.Tensor:
        """model.py:133-165: tokens (B, L) int -> logits (B, L, vocab)."""
        tokens = torch.as_tensor(np.asarray(tokens)) if isinstance(tokens, np.ndarray) else tokens
        seq_len = int(tokens.shape[1])
        if seq_len == 0:
            raise ValueError("prefill requires at least one token")
        self._validate_prefill_bounds(cache, seq_len)
        chunk_size = max(1, min(self.config.hot_capacity, seq_len))
        out: List[torch.Tensor] = []
        chunk_start = 0
        while chunk_start < seq_len:
            chunk_end = min(seq_len, chunk_start + chunk_size)
            start_pos = self._context_end(cache)
            x = self._embed(tokens[:, chunk_start:chunk_end])
            out.append(self._forward(x, cache, start_pos))
            chunk_start = chunk_end
        return out[0] if len(out) == 1 else torch.cat(out, dim=1)

    def decode_step(self, token_id: ArrayLike, cache: RFSNCache, pos: int) -> torch.Tensor:
        """model.py:167-189: token_id (B,) -> logits (B, vocab).

        When the cache allows it (bf16/f16, head_dim 128, <= 4 query heads per KV
        head, every archived block resident in HBM, no prefetch in flight) the
        step replays a CUDA graph of the whole network, captured once and again
        after every page-table change; the host only runs the cache bookkeeping.
        Otherwise (or with ``use_graphs = False``) it runs op by op."""
        self._validate_decode_bounds(cache, pos)
        token_id = torch.as_tensor(np.asarray(token_id)) if isinstance(token_id, np.ndarray) else token_id
        if self.use_graphs:
            if self._graph is None or self._graph.cache is not cache:
                self._graph = _DecodeGraph(self, cache) if _DecodeGraph.supported(self, cache) else None
            if self._graph is not None and self._graph.eligible():
                return self._graph.step(token_id, pos)
        x = self._embed(token_id.reshape(-1, 1))
        return self._forward(x, cache, pos)[:, 0, :]

    def generate(self, prompt_ids: ArrayLike, max_new_tokens: int, cache: Optional[RFSNCache] = None,
                 temperature: float = 1.0, top_p: float = 1.0, top_k: int = 0, repetition_penalty: float = 1.0,
                 generator: Optional[torch.Generator] = None) -> List[torch.Tensor]:
        """model.py:191-264: prefill, then ``max_new_tokens - 1`` decode steps."""
        prompt_ids = torch.as_tensor(np.asarray(prompt_ids)) if isinstance(prompt_ids, np.ndarray) else prompt_ids
        B, L = int(prompt_ids.shape[0]), int(prompt_ids.shape[1])
        if cache is None:
            cache = RFSNCache(self.config, batch_size=B, device=self.device)
        cfg = self.config
        requested_total = self._context_end(cache) + L + max_new_tokens
        if cfg.max_position_embeddings > 0 and requested_total > cfg.max_position_embeddings:
            raise ValueError(
                "Prompt plus requested generation would exceed "
                f"max_position_embeddings={cfg.max_position_embeddings}"
            )
        if cfg.runtime_mode == RuntimeMode.EXACT and requested_total > cfg.hot_capacity:
            raise RuntimeError(
                "runtime_mode='exact' is hot-window only; prompt plus requested generation would exceed "
                f"hot_capacity={cfg.hot_capacity}"
            )
        seen = prompt_ids.to(self.device, torch.long)
        logits = self.prefill(prompt_ids, cache)
        nxt = self._sample(logits[:, -1, :], temperature, top_p, top_k, repetition_penalty, seen, generator)
        generated = [nxt]
        seen = torch.cat([seen, nxt[:, None].long()], dim=1)
        pos = L
        for _ in range(max_new_tokens - 1):
            logits = self.decode_step(nxt, cache, pos)
            nxt = self._sample(logits, temperature, top_p, top_k, repetition_penalty, seen, generator)
            generated.append(nxt)
            seen = torch.cat([seen, nxt[:, None].long()], dim=1)
            pos += 1
        return generated

    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float, top_p: float, top_k: int, repetition_penalty: float,
                seen_ids: torch.Tensor, generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """model.py:266-336: greedy at temperature 0, else repetition penalty,
        top-k, temperature, top-p (nucleus) and a categorical draw."""
        if temperature == 0.0:
            return torch.argmax(logits, dim=-1).to(torch.int32)
        logits = logits.float()
        if repetition_penalty != 1.0:
            mask = torch.zeros_like(logits)
            mask.scatter_(1, seen_ids.long(), 1.0)
            factor = mask * (repetition_penalty - 1.0) + 1.0
            logits = torch.where(logits > 0, logits / factor, logits * factor)
        if top_k > 0:
            threshold = torch.topk(logits, top_k, dim=-1).values[:, -1:]
            logits = torch.where(logits >= threshold, logits, torch.full_like(logits, float("-inf")))
        scaled = logits / temperature
        if top_p < 1.0:
            probs = torch.softmax(scaled, dim=-1)
            sorted_probs, sorted_idx = torch.sort(probs, dim=-1, descending=True)
            cumsum = torch.cumsum(sorted_probs, dim=-1)
            keep = (cumsum - sorted_probs) < top_p
            sorted_probs = sorted_probs * keep
            sorted_probs = sorted_probs / sorted_probs.sum(dim=-1, keepdim=True)
            local = torch.multinomial(sorted_probs, 1, generator=generator)
            return torch.gather(sorted_idx, 1, local)[:, 0].to(torch.int32)
        probs = torch.softmax(scaled, dim=-1)
        return torch.multinomial(probs, 1, generator=generator)[:, 0].to(torch.int32)


class _DecodeGraph:
    """The decode step of a whole model as one CUDA graph.

    Per step the host runs each layer's cache bookkeeping exactly as
    ``attention_step`` would (seal rule, append counters, prefetch hook,
    segment walk with its LRU touches) and writes the step state (position,
    ring write index, hot window) to device memory; the graph then embeds the
    token, runs every layer with the fused RoPE/append and the decode kernel
    reading that state, and writes the logits. The page tables, arena
    descriptors and workspace are captured by value, so the graph is captured
    again whenever one of them changes (a seal, a promotion, an arena growth)."""

    RING = 8  # pinned step-state buffers in flight

    @staticmethod
    def supported(model: "RFSNModel", cache: RFSNCache) -> bool:
        cfg = model.config
        return (model.device.type == "cuda" and model.dtype in (torch.bfloat16, torch.float16)
                and cfg.head_dim == 128 and cfg.num_heads // cfg.num_kv_heads <= 4
                and all(lc.dtype == model.dtype for lc in cache.layers))

    def __init__(self, model: "RFSNModel", cache: RFSNCache) -> None:
        self.model = model
        self.cache = cache
        dev = model.device
        self.tok = torch.zeros((0,), dtype=torch.long, device=dev)
        self.state_dev = torch.zeros(native.STEP_STATE_LEN, dtype=torch.int32, device=dev)
        self.state_host = [torch.zeros(native.STEP_STATE_LEN, dtype=torch.int32).pin_memory() for _ in range(self.RING)]
        self.state_done = [torch.cuda.Event() for _ in range(self.RING)]
        self.n = 0
        self.workspace = native.Workspace(dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.key = None
        self.logits: Optional[torch.Tensor] = None
        self.replays = 0
        self.captures = 0

    def eligible(self) -> bool:
        layers = self.cache.layers
        first = (layers[0].hot_head_index, layers[0].hot_seq_len, layers[0].hot_start)
        for lc in layers:
            if lc.residency_manager.has_pending or not lc.all_blocks_resident():
                return False
            if (lc.hot_head_index, lc.hot_seq_len, lc.hot_start) != first:
                return False
        return True

    def step(self, token_id: torch.Tensor, pos: int) -> torch.Tensor:
        model, cache = self.model, self.cache
        segs, write_index = [], None
        for lc in cache.layers:
            # attention_step's host part for one token (layer.py:134-139)
            lc.evict_for_append(1)
            wi = lc.hot_write_index
            lc._check_append(1)
            lc.hot_seq_len += 1
            lc.maybe_prefetch_for_decode(pos)
            sg = lc.get_attention_segments()
            segs.append(sg)
            write_index = wi
        head, hlen, hstart = segs[0].hot_state
        slot = self.n % self.RING
        self.n += 1
        self.state_done[slot].synchronize()  # the copy that last read this buffer has run
        self.state_host[slot].copy_(torch.tensor([pos, write_index, head, hlen, hstart, 0, 0, 0], dtype=torch.int32))
        self.state_dev.copy_(self.state_host[slot], non_blocking=True)
        self.state_done[slot].record()
        B = int(token_id.numel())
        key = (B,) + tuple((lc.arena.handle.value if hasattr(lc.arena.handle, "value") else id(lc.arena),
                            lc._arena_k.data_ptr(), sg.table[0].data_ptr() if sg.table is not None else 0,
                            sg.table[1:] if sg.table is not None else None) for lc, sg in zip(cache.layers, segs))
        if self.tok.numel() != B:
            self.tok = torch.zeros((B,), dtype=torch.long, device=model.device)
        self.tok.copy_(token_id.reshape(-1).to(device=model.device, dtype=torch.long), non_blocking=True)
        if key != self.key or self.graph is None:
            self._capture(segs)
            self.key = key
            self.captures += 1
        else:
            self.graph.replay()
            self.replays += 1
        return self.logits.clone()

    def _forward(self, segs) -> torch.Tensor:
        model, cache = self.model, self.cache
        x = F.embedding(self.tok.view(-1, 1), model.params["embed_tokens.weight"])
        for i, layer in enumerate(model.layers):
            lc, sg = cache.layer(i), segs[i]
            x = layer(x, lc, attn=lambda q, k, v, lc=lc, sg=sg: self._attention(lc, sg, q, k, v))
        x = _layer_norm(x, model.params["norm.weight"], model.params["norm.bias"], model.config.norm_eps)
        return model._lm_head(x)[:, 0, :]

    def _attention(self, lc, segs, q, k, v) -> torch.Tensor:
        B, H, L, D = (int(t) for t in q.shape)
        qc, kc, vc = _as(q, lc.device, lc.dtype), _as(k, lc.device, lc.dtype), _as(v, lc.device, lc.dtype)
        q_rot = torch.empty((B, H, L, D), dtype=torch.float32, device=lc.device)
        native.check(
            native.lib().rfsn_rope_append_step(
                qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), native.dtype_code(lc.dtype), lc.inv_freq().data_ptr(),
                self.state_dev.data_ptr(), None, B, H, lc.num_kv_heads, L, D, q_rot.data_ptr(), lc.arena.handle, 0,
                lc.config.hot_capacity, native.stream_ptr()),
            "rfsn_rope_append_step",
        )
        return paged_attention(lc, q_rot, 0, segs, workspace=self.workspace, step_state=self.state_dev)

    def _capture(self, segs) -> None:
        """Run this step once op by op on a side stream (the warm-up torch asks
        for before a capture; it also produces this step's result), then capture."""
        model = self.model
        ws_bytes = native.workspace_bytes(int(self.tok.numel()), model.config.num_heads, model.config.num_kv_heads, 1,
                                          model.config.head_dim, 0)
        self.workspace.get(ws_bytes)
        side = self.stream
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            logits = self._forward(segs)
        torch.cuda.current_stream().wait_stream(side)
        logits.record_stream(torch.cuda.current_stream())  # read below on this stream
        self.graph = None
        out = {}
        self.graph = capture_graph(lambda: out.setdefault("logits", self._forward(segs)), side)
        self.logits = out["logits"]
        # the capture recorded work without running it: this step's result is the warm-up's
        self.logits.copy_(logits)


RFSNMLX = RFSNModel  # the reference's class names
RFSNLayerMLX = RFSNLayer
