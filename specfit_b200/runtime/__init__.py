"""Drop-in runtime of the MoE verification path (reference: specfit.runtime)."""
from .cache_observer import CacheTransition, CacheTransitionObserver, RecordingCacheTransitionObserver
from .cache_snapshot import CacheSlotSnapshot, GpuExpertCacheSnapshot, PendingTransferSnapshot
from .gpu_expert_cache import GpuExpertCache
from .lease import ExpertCacheStats, ExpertLease, NoEvictableSlotError
from .moe_block import Qwen3B200SparseMoeBlock, Qwen3B200TopKRouter
from .qwen3_expert_prefetch import Qwen3ExpertPrefetch
from .qwen3_loader import load_offloaded_qwen3
from .qwen3_offloaded_experts import ExpertExecutionPolicy, Qwen3OffloadedExperts, ReductionMode
from .state import ExpertKey, RuntimeEventKind

__all__ = [
    "CacheSlotSnapshot", "CacheTransition", "CacheTransitionObserver", "ExpertCacheStats",
    "ExpertExecutionPolicy", "ExpertKey", "ExpertLease", "GpuExpertCache", "GpuExpertCacheSnapshot",
    "NoEvictableSlotError", "PendingTransferSnapshot", "Qwen3B200SparseMoeBlock",
    "Qwen3B200TopKRouter", "Qwen3ExpertPrefetch", "Qwen3OffloadedExperts",
    "RecordingCacheTransitionObserver",
    "ReductionMode", "RuntimeEventKind", "load_offloaded_qwen3",
]
