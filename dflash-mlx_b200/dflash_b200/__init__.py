"""dflash-b200: the DFlash speculative draft/verify hot path on NVIDIA B200 (sm_100a).

Public surface mirrors the reference package's ``__all__`` (dflash_mlx/__init__.py:1-22).
"""
from .adapters import LoadedTargetModel, adapter_for_model_type, load_target_model
from .api import DFlashGenerator, DFlashResult, DFlashStreamEvent, load_draft_model
from .model import DraftModel as DFlashDraftModel
from .runtime import dflash_generate, dflash_generate_stream, longest_prefix_match, sample_tokens

__all__ = [
    "DFlashGenerator",
    "DFlashResult",
    "DFlashStreamEvent",
    "DFlashDraftModel",
    "LoadedTargetModel",
    "adapter_for_model_type",
    "dflash_generate",
    "dflash_generate_stream",
    "load_draft_model",
    "load_target_model",
    "longest_prefix_match",
    "sample_tokens",
]
