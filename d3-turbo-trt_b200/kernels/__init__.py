"""sm_100a attention kernels (mirrors d3trt/kernels)."""
