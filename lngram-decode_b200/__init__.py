"""lngram_b200: the Lngram v2 route n-gram memory lookup on B200 (sm_100a).

A drop-in, inference-only replacement for the reference's memory modules
(``ffnmem/memory/lngram_v2.py``, ``ffnmem/memory/wrapper.py``) and its per-token drafter
(``drafting/cpu/drafter.cpp``, ``drafting/cpu_drafter.py``), backed by hand-written CUDA kernels
behind the C ABI of ``include/lngram_b200.h``.  There is no CPU fallback.
"""

from . import _lib
from .bundle import Bundle, load_bundle, read_header, write_bundle
from .drafter import DraftOut, Drafter, GpuDrafter, OnlineCounts, make_drafter
from .memory import LngramIncrementalState, LngramMemory, RouteNgramMemoryV2, rms_norm

__all__ = ["Bundle", "DraftOut", "Drafter", "GpuDrafter", "LngramIncrementalState", "OnlineCounts", "LngramMemory", "RouteNgramMemoryV2", "_lib", "load_bundle",
           "make_drafter", "read_header", "rms_norm", "write_bundle"]
from .seams import MemoryCache, ancestor_table, decode_memory_step, memory_step, tree_memory_block, tree_ngram_codes, tree_slots  # noqa: E402

__all__ += ["MemoryCache", "ancestor_table", "decode_memory_step", "memory_step", "tree_memory_block", "tree_ngram_codes", "tree_slots"]
from . import serving, sharded  # noqa: E402
from .sharded import RouteShardedMemory  # noqa: E402

__all__ += ["RouteShardedMemory", "serving", "sharded"]
