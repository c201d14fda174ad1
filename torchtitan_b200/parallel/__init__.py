from .parallel_dims import ParallelDims

__all__ = ["ParallelDims"]
