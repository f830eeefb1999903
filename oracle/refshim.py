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
    (custom_qwen35_model.py:1029-1074) uses mx.concatenate / mx.repeat.

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
    mx.fast = types.SimpleNamespace(metal_kernel=lambda **k: None)
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
    for name in ("Linear", "RMSNorm", "Embedding", "Conv1d"):
        setattr(nn, name, type(name, (_Module,), {}))
    nn.silu = lambda x: x / (1.0 + np.exp(-x))
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
    base.scaled_dot_product_attention = lambda *a, **k: None
    gd = types.ModuleType("mlx_lm.models.gated_delta")
    for n in ("compute_g", "gated_delta_kernel", "gated_delta_ops", "gated_delta_update"):
        setattr(gd, n, lambda *a, **k: (_ for _ in ()).throw(NotImplementedError(n)))
    q3 = types.ModuleType("mlx_lm.models.qwen3")
    q3.MLP = type("MLP", (_Module,), {})
    q3.create_attention_mask = lambda *a, **k: None
    q35 = types.ModuleType("mlx_lm.models.qwen3_5")
    qn = types.ModuleType("mlx_lm.models.qwen3_next")
    for n in ("Qwen3NextAttention", "Qwen3NextMLP", "Qwen3NextRMSNormGated", "Qwen3NextSparseMoeBlock"):
        setattr(qn, n, type(n, (_Module,), {}))
    rope = types.ModuleType("mlx_lm.models.rope_utils")
    rope.initialize_rope = lambda *a, **k: None
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
