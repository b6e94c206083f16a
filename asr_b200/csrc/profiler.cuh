// Per-kernel CUDA-event timing of this library's own launches (diagnostics).
// When enabled through asr_profiler_enable, every launch site wrapped in a
// KernelTimer records a start and a stop event on the launching stream; the
// report sums the elapsed device time per kernel name. Each KernelTimer, and
// each entry point (NvtxRange), is also an NVTX range of the same name, so a
// timeline profiler shows the op and kernel structure; without a profiler
// attached the NVTX calls do nothing.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

namespace asr {

// NVTX range over a scope (an op entry point).
class NvtxRange {
  public:
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

class KernelTimer {
  public:
    KernelTimer(const char* name, cudaStream_t stream);
    ~KernelTimer();
    KernelTimer(const KernelTimer&) = delete;
    KernelTimer& operator=(const KernelTimer&) = delete;

  private:
    const char* name_;
    cudaStream_t stream_;
    cudaEvent_t start_ = nullptr;
};

}  // namespace asr
