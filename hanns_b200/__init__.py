"""hanns_b200 -- B200-native (sm_100a) IVF-USQ batched search behind Hanns' API.

The compute lives in hanns_b200/lib/libhanns_gpu.so (CUDA kernels + C ABI, see
include/hanns_gpu.h).  This package is the Python mirror of the reference's
IvfUsqIndex API over that C ABI.
"""
from .ivf_usq import (FILTER_FUSED, FILTER_NONE, FILTER_POST, METRIC_IP, METRIC_L2, IvfUsqConfig,
                      IvfUsqIndex, SearchRequest, SearchResult)

__all__ = ["IvfUsqConfig", "IvfUsqIndex", "SearchRequest", "SearchResult", "METRIC_L2", "METRIC_IP",
           "FILTER_NONE", "FILTER_POST", "FILTER_FUSED"]
