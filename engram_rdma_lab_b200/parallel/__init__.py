from .dist import assigned_devices, bind_rank, gather_floats, init_dist, max_over_ranks

__all__ = ["assigned_devices", "bind_rank", "gather_floats", "init_dist", "max_over_ranks"]
