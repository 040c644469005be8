from .perf import compare_memory_kernel_perf, perf_cuda

__all__ = ["perf_cuda", "compare_memory_kernel_perf"]
