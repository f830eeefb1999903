"""Numpy stand-in for the ``mlx`` / ``mlx_lm`` / ``huggingface_hub`` imports of the
reference package — TEST INFRASTRUCTURE ONLY (golden-fixture generation).

MLX is not installable in this container (no Apple Metal, no wheel, no
network). The reference modules this build pins against only use a small,
numpy-compatible subset of ``mlx.core`` on the code paths exercised:

  * dflash_mlx/runtime.py (decode loop, accept, commit, stop; runtime.py:22-589)
    uses mx.array / mx.uint32 / mx.eval / mx.argmax / .tolist() / .item();
  * dflash_mlx/adapters.py ``advance_gated_delta_states`` CPU branch
    (adapters.py:93-135) uses astype / broadcasting / mx.sum;
  * dflash_mlx/custom_qwen35_model.py ``rollback_linear_caches``
    (custom_qwen35_model.py:1029-1074) uses mx.concatenate / mx.repeat;
  * dflash_mlx/draft.py ``DFlashDraftModel`` (draft.py:68-223) runs on numpy
    restatements of the layers it builds from: ``nn.Linear`` (y = x W^T + b),
    ``nn.RMSNorm`` (w * x / sqrt(mean(x^2) + eps)), mlx-lm ``qwen3.MLP``
    (down(silu(gate(x)) * up(x))), ``rope_utils.initialize_rope`` with
    traditional=False (rotation of the two halves of the first ``dims`` features by
    position * base^(-2i/dims)), ``base.scaled_dot_product_attention`` (GQA softmax
    attention; mask "causal" aligned to the last key) and ``cache.KVCache``
    (append along the sequence axis, ``offset``, ``trim``);
  * dflash_mlx/custom_qwen35_model.py ``forward_linear_layer_explicit_with_record``
    and ``forward_full_attention_layer_explicit`` (custom_qwen35_model.py:409-540)
    additionally use ``mx.split``, ``mx.fast.rms_norm``,
    ``mx.fast.scaled_dot_product_attention`` and mlx-lm's ``gated_delta.compute_g``
    (g = exp(-exp(A_log) * softplus(a + dt_bias))), ``gated_delta.gated_delta_ops``
    (per token: S <- g S; S <- S + beta (v - S k) k^T; y = S q, q / k repeated to the
    value heads) and the depthwise ``nn.Conv1d`` (weight [C, K, 1], no padding), all
    restated here in numpy.

``install()`` registers stub modules so that those reference files import
unchanged from the read-only reference tree; ``import_reference(root)`` loads
them as the package ``dflash_mlx`` without running its ``__init__`` (which pulls
in the CLI and HTTP server). Nothing here is used by the product.
"""
from __future__ import annotations

import importlib
import sys
import types

import numpy as np


def _sdpa(queries, keys, values, cache=None, scale=1.0, mask=None):
    """Softmax attention, q [B, Hq, L, D] against k / v [B, Hkv, S, D] (GQA repeat);
    mask "causal" lets query i see keys up to S - L + i."""
    rep = queries.shape[1] // keys.shape[1]
    k = np.repeat(keys, rep, axis=1)
    v = np.repeat(values, rep, axis=1)
    s = queries @ np.swapaxes(k, -1, -2) * scale
    if mask == "causal":
        L, S = s.shape[-2], s.shape[-1]
        allowed = np.arange(S)[None, :] <= (S - L + np.arange(L))[:, None]
        s = np.where(allowed, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    return (p / p.sum(axis=-1, keepdims=True)) @ v


class _Module:
    """Base class stand-in for mlx.nn.Module (only subclassed at import time)."""

    def __init__(self, *a, **k):
        pass


def _make_core() -> types.ModuleType:
    mx = types.ModuleType("mlx.core")
    mx.uint32 = np.uint32
    mx.int32 = np.int32
    mx.float32 = np.float32
    mx.float16 = np.float16
    mx.bfloat16 = np.float32  # only used as a dtype tag on the stubbed paths
    class array:  # noqa: N801 - a type, so that ``mx.array | None`` annotations evaluate
        def __new__(cls, x, dtype=None):
            return np.array(x, dtype=dtype)

    mx.array = array
    mx.eval = lambda *a, **k: None
    mx.argmax = lambda x, axis=None: np.argmax(x, axis=axis)
    mx.sum = lambda x, axis=None, keepdims=False: np.sum(x, axis=axis, keepdims=keepdims)
    mx.concatenate = lambda xs, axis=0: np.concatenate(xs, axis=axis)
    mx.repeat = lambda x, r, axis=None: np.repeat(x, r, axis=axis)
    mx.zeros = lambda shape, dtype=np.float32: np.zeros(shape, dtype=dtype)
    mx.exp = np.exp
    mx.log = np.log
    mx.sigmoid = lambda x: 1.0 / (1.0 + np.exp(-x))
    mx.where = np.where
    mx.get_peak_memory = lambda: 0
    mx.reset_peak_memory = lambda: None
    mx.gpu = "gpu"
    mx.cpu = "cpu"
    mx.default_device = lambda: "cpu"
    mx.set_default_device = lambda d: None
    metal = types.SimpleNamespace(is_available=lambda: False)
    mx.metal = metal
    rnd = types.SimpleNamespace(seed=lambda s: None, uniform=lambda **k: np.zeros(k.get("shape", (1,))),
                                categorical=lambda *a, **k: (_ for _ in ()).throw(NotImplementedError()))
    mx.random = rnd
    mx.compile = lambda f: f
    def rms_norm(x, w, eps):
        y = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
        return y if w is None else w * y

    def fast_sdpa(queries, keys, values, scale=1.0, mask=None):
        return _sdpa(queries, keys, values, scale=scale, mask=mask)

    mx.fast = types.SimpleNamespace(metal_kernel=lambda **k: None, rms_norm=rms_norm,
                                    scaled_dot_product_attention=fast_sdpa)
    mx.split = lambda x, idx, axis=0: np.split(x, idx, axis=axis)
    return mx


def install() -> None:
    if "mlx.core" in sys.modules and getattr(sys.modules["mlx.core"], "_dflash_shim", False):
        return
    mx = _make_core()
    mx._dflash_shim = True
    mlx = types.ModuleType("mlx")
    mlx.core = mx
    nn = types.ModuleType("mlx.nn")
    nn.Module = _Module
    nn.Embedding = type("Embedding", (_Module,), {})

    class Conv1d(_Module):  # depthwise (groups == channels), no padding: [B, L, C] -> [B, L - K + 1, C]
        def __init__(self, in_channels, out_channels, kernel_size, groups=1, bias=False, padding=0):
            self.weight = np.zeros((out_channels, kernel_size, in_channels // groups))
            self.groups = groups

        def __call__(self, x):
            K = self.weight.shape[1]
            L = x.shape[1] - K + 1
            return sum(x[:, j:j + L, :] * self.weight[:, j, 0] for j in range(K))

    nn.Conv1d = Conv1d
    nn.silu = lambda x: x / (1.0 + np.exp(-x))

    class Linear(_Module):
        def __init__(self, input_dims, output_dims, bias=True):
            self.weight = np.zeros((output_dims, input_dims))
            self.bias = np.zeros(output_dims) if bias else None

        def __call__(self, x):
            y = x @ self.weight.T
            return y + self.bias if self.bias is not None else y

    class RMSNorm(_Module):
        def __init__(self, dims, eps=1e-5):
            self.weight = np.ones(dims)
            self.eps = eps

        def __call__(self, x):
            return self.weight * x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + self.eps)

    nn.Linear, nn.RMSNorm = Linear, RMSNorm
    layers = types.ModuleType("mlx.nn.layers")
    dist = types.ModuleType("mlx.nn.layers.distributed")
    dist.shard_inplace = dist.shard_linear = dist.sum_gradients = lambda *a, **k: None
    mlx_utils = types.ModuleType("mlx.utils")
    mlx_utils.tree_map = lambda f, t: t
    mlx.nn = nn
    mlx.utils = mlx_utils

    hub = types.ModuleType("huggingface_hub")
    hub.snapshot_download = lambda *a, **k: (_ for _ in ()).throw(RuntimeError("no network"))

    lm = types.ModuleType("mlx_lm")
    lm.load = lambda *a, **k: (_ for _ in ()).throw(RuntimeError("no checkpoints"))
    models = types.ModuleType("mlx_lm.models")
    cache = types.ModuleType("mlx_lm.models.cache")

    class KVCache:
        def __init__(self):
            self.offset = 0
            self.keys = None
            self.values = None

        def update_and_fetch(self, keys, values):  # [B, H, S, D], appended after offset
            if self.keys is None:
                self.keys, self.values = keys, values
            else:
                self.keys = np.concatenate([self.keys[..., :self.offset, :], keys], axis=2)
                self.values = np.concatenate([self.values[..., :self.offset, :], values], axis=2)
            self.offset += keys.shape[2]
            return self.keys, self.values

        def trim(self, n):
            n = min(self.offset, n)
            self.offset -= n
            return n

    class ArraysCache(list):
        def __init__(self, size=2):
            super().__init__([None] * size)

        @property
        def cache(self):
            return list(self)

    cache.KVCache = KVCache
    cache.ArraysCache = ArraysCache
    base = types.ModuleType("mlx_lm.models.base")

    class BaseModelArgs:
        pass

    base.BaseModelArgs = BaseModelArgs
    base.create_attention_mask = lambda *a, **k: None
    base.create_ssm_mask = lambda *a, **k: None
    base.scaled_dot_product_attention = _sdpa
    gd = types.ModuleType("mlx_lm.models.gated_delta")
    for n in ("gated_delta_kernel", "gated_delta_update"):
        setattr(gd, n, lambda *a, **k: (_ for _ in ()).throw(NotImplementedError(n)))

    def compute_g(A_log, a, dt_bias):
        x = a + dt_bias
        return np.exp(-np.exp(A_log) * np.logaddexp(0.0, x))

    def gated_delta_ops(q, k, v, g, beta, state=None, mask=None):
        # q, k [B, T, Hk, Dk]; v [B, T, Hv, Dv]; g, beta [B, T, Hv]; state [B, Hv, Dv, Dk]
        B, T, Hk, Dk = k.shape
        Hv, Dv = v.shape[2], v.shape[3]
        q = np.repeat(q, Hv // Hk, axis=2)
        k = np.repeat(k, Hv // Hk, axis=2)
        S = np.zeros((B, Hv, Dv, Dk)) if state is None else np.array(state, dtype=np.float64)
        ys = []
        for t in range(T):
            S = S * g[:, t, :, None, None]
            kv = np.einsum("bhvk,bhk->bhv", S, k[:, t])
            delta = (v[:, t] - kv) * beta[:, t, :, None]
            S = S + np.einsum("bhv,bhk->bhvk", delta, k[:, t])
            ys.append(np.einsum("bhvk,bhk->bhv", S, q[:, t]))
        return np.stack(ys, axis=1), S

    gd.compute_g, gd.gated_delta_ops = compute_g, gated_delta_ops
    q3 = types.ModuleType("mlx_lm.models.qwen3")
    class MLP(_Module):
        def __init__(self, dim, hidden_dim):
            self.gate_proj = Linear(dim, hidden_dim, bias=False)
            self.up_proj = Linear(dim, hidden_dim, bias=False)
            self.down_proj = Linear(hidden_dim, dim, bias=False)

        def __call__(self, x):
            g = self.gate_proj(x)
            return self.down_proj(g / (1.0 + np.exp(-g)) * self.up_proj(x))

    q3.MLP = MLP
    q3.create_attention_mask = lambda *a, **k: None
    q35 = types.ModuleType("mlx_lm.models.qwen3_5")
    qn = types.ModuleType("mlx_lm.models.qwen3_next")
    for n in ("Qwen3NextAttention", "Qwen3NextSparseMoeBlock"):
        setattr(qn, n, type(n, (_Module,), {}))

    class RMSNormGated(_Module):  # rms_norm(x) * w, then silu(gate) * that
        def __init__(self, dims, eps=1e-6):
            self.weight = np.ones(dims)
            self.eps = eps

        def __call__(self, x, gate=None):
            y = self.weight * x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + self.eps)
            return y if gate is None else gate / (1.0 + np.exp(-gate)) * y

    qn.Qwen3NextRMSNormGated = RMSNormGated
    qn.Qwen3NextMLP = q3.MLP
    rope = types.ModuleType("mlx_lm.models.rope_utils")
    class RoPE:
        def __init__(self, dims, base=10000.0, traditional=False, scaling_config=None, max_position_embeddings=None):
            if traditional or scaling_config:
                raise NotImplementedError("only plain non-traditional RoPE is restated")
            self.dims, self.base = dims, base

        def __call__(self, x, offset=0):  # x [..., L, D]
            half = self.dims // 2
            inv = self.base ** (-np.arange(0, self.dims, 2) / self.dims)
            ang = (offset + np.arange(x.shape[-2]))[:, None] * inv[None, :]
            c, s = np.cos(ang), np.sin(ang)
            x1, x2 = x[..., :half], x[..., half:self.dims]
            return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s, x[..., self.dims:]], axis=-1)

    rope.initialize_rope = lambda dims, base=10000.0, traditional=False, scaling_config=None, \
        max_position_embeddings=None: RoPE(dims, base, traditional, scaling_config, max_position_embeddings)
    utils = types.ModuleType("mlx_lm.utils")
    utils.quantize_model = lambda *a, **k: (None, {})
    gen = types.ModuleType("mlx_lm.generate")
    gen.wired_limit = lambda model: __import__("contextlib").nullcontext()
    for name, mod in {
        "mlx": mlx, "mlx.core": mx, "mlx.nn": nn, "mlx.nn.layers": layers, "mlx.nn.layers.distributed": dist,
        "mlx.utils": mlx_utils, "huggingface_hub": hub, "mlx_lm": lm, "mlx_lm.models": models,
        "mlx_lm.models.cache": cache, "mlx_lm.models.base": base, "mlx_lm.models.gated_delta": gd,
        "mlx_lm.models.qwen3": q3, "mlx_lm.models.qwen3_5": q35, "mlx_lm.models.qwen3_next": qn,
        "mlx_lm.models.rope_utils": rope, "mlx_lm.utils": utils, "mlx_lm.generate": gen,
    }.items():
        sys.modules[name] = mod
    models.cache, models.base, models.gated_delta = cache, base, gd
    models.qwen3, models.qwen3_5, models.qwen3_next, models.rope_utils = q3, q35, qn, rope


def import_reference(root: str, modules=("runtime", "adapters", "custom_qwen35_model")) -> dict:
    """Imports reference modules from ``root``/dflash_mlx under the shim."""
    install()
    sys.dont_write_bytecode = True
    pkg = types.ModuleType("dflash_mlx")
    pkg.__path__ = [f"{root}/dflash_mlx"]
    sys.modules["dflash_mlx"] = pkg
    return {m: importlib.import_module(f"dflash_mlx.{m}") for m in modules}
