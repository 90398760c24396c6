"""tidegs_b200: B200-native (sm_100a) resident-block optimizer, slot
materialization and dirty write-back for TideGS.

Drop-in classes (same names and behaviour as the reference's):
    GPUResidentAdam                      strategies/tide_engine/gpu_resident_optimizer.py
    SelectiveAdam, ResidentAdamContext   optimizer.py
    DoubleBufferGPUWorkingSet, GPUBuffer strategies/tide_engine/double_buffer_gpu.py
    GPUWorkingSet, PendingBlockWriteback strategies/tide_engine/gpu_working_set.py
    SparseGradAccumulator                strategies/tide_engine/engine.py:1793-1826, 2434-2471
    PinnedBlockCache, BlockLogStore,     storage/tiered_cache_manager.py,
    CachedBlockReader                    storage/log_storage_manager.py, storage/block_reader.py
    BlockCuller                          storage/gaussian_block.py (FrustumCuller)
    compute_topc_resident_transition,    strategies/tide_engine/resident_policy.py
    compute_passthrough_resident_transition
    render.fully_fused_projection,       gsplat 1.0.0 (the engine's render path,
    render.isect_tiles, isect_offset_encode, strategies/tide_engine/engine.py:481-561)
    render.rasterize_to_pixels
plus SelectiveSophia (no reference counterpart) and PinnedBlockPool.

All device work runs in libtidegs_b200.so (include/tidegs_b200.h); importing
the package does not touch the GPU, and constructing any class that owns
device memory requires CUDA and the built library. The host-tier classes are
host code (page-locked memory when CUDA is present) whose device transfers
are issued by GPUWorkingSet and DoubleBufferGPUWorkingSet.
"""
from .culling import BlockCuller
from .resident_policy import (RecencyScores, ResidentTransition,
                              compute_passthrough_resident_transition,
                              compute_topc_resident_transition)
from .block_reader import (BlockBatch, BlockLayout, BlockReader, PinnedBlockPool,
                           UnifiedParamsBlockReader, parse_block_row_components)
from .double_buffer_gpu import DoubleBufferGPUWorkingSet, GPUBuffer, ResidentHandoffResult
from .gpu_resident_optimizer import GPUResidentAdam
from .gpu_working_set import (GPUWorkingSet, PendingBlockBounds, PendingBlockWriteback,
                              PendingCacheWriteback)
from .host_tier import BlockLogStore, CachedBlockReader, PinnedBlockCache
from .optimizer import ResidentAdamContext, SelectiveAdam, SelectiveSophia
from .sparse_grad import SparseGradAccumulator

__all__ = [
    "BlockBatch", "BlockLayout", "BlockReader", "PinnedBlockPool", "UnifiedParamsBlockReader",
    "parse_block_row_components", "DoubleBufferGPUWorkingSet", "GPUBuffer",
    "ResidentHandoffResult", "GPUResidentAdam", "GPUWorkingSet", "PendingBlockBounds",
    "PendingBlockWriteback", "ResidentAdamContext", "SelectiveAdam", "SelectiveSophia",
    "SparseGradAccumulator", "PendingCacheWriteback", "BlockLogStore", "CachedBlockReader",
    "PinnedBlockCache", "BlockCuller", "RecencyScores", "ResidentTransition",
    "compute_passthrough_resident_transition", "compute_topc_resident_transition",
]
