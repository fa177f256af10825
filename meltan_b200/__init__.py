"""meltan_b200 -- B200-native search hot path for MetalANNS.

The exact flat scan with top-k, IVF-flat probe-and-scan and IVF-PQ ADC scoring
run as hand-written sm_100a CUDA kernels in ``libmans_cuda.so`` behind the C
ABI of ``include/mans_cuda.h``; this package is the host-side binding.
"""
from .core import (  # noqa: F401
    ANNSError,
    ConstructionFailed,
    CorruptFile,
    MannInfo,
    Context,
    DeviceNotSupported,
    DimensionMismatch,
    EMPTY_ID,
    FlatGPUSearch,
    GPUExecutionFailed,
    GPUPipelineUnavailable,
    GPUResourceExhausted,
    MAX_TOP_K,
    Metric,
    SearchFailed,
    SearchResult,
    TC_AUTO,
    TC_BF16,
    TC_INT8,
    VectorBuffer,
    Workspace,
    check,
    mann_info,
    topk_merge_device,
)
from .ivf import IVFFlatSearch, Partition, assign_rows  # noqa: F401,E402
from .pq import GPUADCSearch, IVFPQIndex  # noqa: F401,E402
from .pq import encode as pq_encode  # noqa: F401,E402
from . import train  # noqa: F401,E402
from . import shard  # noqa: F401,E402
from .shard import (ShardedFlatSearch, ShardedIVFPQSearch, ShardedIVFSearch,  # noqa: F401,E402
                    row_shard)
