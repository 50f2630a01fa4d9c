from .dist import LOCAL, DistContext, all_reduce_sum_, barrier, gather_rows, init_from_env

__all__ = ["DistContext", "LOCAL", "all_reduce_sum_", "barrier", "gather_rows", "init_from_env"]
