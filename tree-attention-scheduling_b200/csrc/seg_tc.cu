// Segment attention for large groups on the 5th-generation tensor cores.
#include "ta_common.cuh"
#include "ta_kernels.cuh"

namespace ta {

cudaError_t launch_seg_tc(const SegParams&, int, int, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace ta
