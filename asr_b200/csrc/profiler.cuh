// Per-kernel CUDA-event timing of this library's own launches (diagnostics).
// When enabled through asr_profiler_enable, every launch site wrapped in a
// KernelTimer records a start and a stop event on the launching stream; the
// report sums the elapsed device time per kernel name.
#pragma once

#include <cuda_runtime.h>

namespace asr {

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
