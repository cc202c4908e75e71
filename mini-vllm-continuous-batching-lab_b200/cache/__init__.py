from .pool import MIN_BLOCKS, KVCachePool, compute_num_gpu_blocks

__all__ = ["KVCachePool", "MIN_BLOCKS", "compute_num_gpu_blocks"]
