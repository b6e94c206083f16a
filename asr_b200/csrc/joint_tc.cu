// bf16 tcgen05 joint network (the tf32 != 0 fast mode). Placeholder until the
// tensor-core kernels land: reports "unsupported" so the fp32 SIMT path runs.
#include "joint.cuh"

namespace asr {

bool tc_supported(const JointArgs&) { return false; }
size_t tc_forward_scratch_bytes(const JointArgs&) { return 0; }
int tc_joint_forward(const JointArgs&, const JointFwdOut&, void*, size_t, cudaStream_t) { return ASR_ERR_UNSUPPORTED; }
size_t tc_backward_scratch_bytes(const JointArgs&, int) { return 0; }
int tc_joint_backward(const JointArgs&, const JointBwdIn&, const JointBwdOut&, int, void*, size_t, cudaStream_t) {
    return ASR_ERR_UNSUPPORTED;
}

}  // namespace asr
