// Allocation-free variant of the TDT forward entry point.
//
// Some callers cannot allocate device memory at the moment they need the loss:
// hosts bound to this library through a bare FFI that own no device allocator,
// services that reserve all GPU memory once at start-up and forbid allocation
// afterwards (real-time or fixed-budget inference), and code that must not let
// a cudaMalloc synchronise the device mid-stream. asr_tdt_forward asks them for
// a workspace; this entry point instead uses a fixed scratch array compiled
// into the library, so the caller passes only its inputs and outputs.
//
// The scratch is one file-scope __device__ array of ASR_TDT_FORWARD_NOALLOC_SCRATCH_BYTES
// bytes; every GPU that loads the library holds it until the process exits.
// Host code cannot use the array's name as a device address. A __device__
// symbol's address belongs to the CUDA context that loaded the module, so it is
// looked up with cudaGetSymbolAddress on every call, in the calling thread's
// current context: any context that has the library loaded works, including a
// primary context re-created after cudaDeviceReset and a driver-API context the
// caller made current. The first call in a context loads the module there (make
// it before any stream capture). All calls share the array and it keeps the last
// call's contents: the lattice bookkeeping kernel rewrites every byte the forward
// reads, so nothing needs clearing, but calls that overlap on the GPU (other
// streams, other host threads) race on it and must be serialised by the caller.
#include "asr_b200.h"

namespace {

static __device__ __align__(256) unsigned char g_tdt_forward_scratch[ASR_TDT_FORWARD_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array in the current context, or nullptr.
void* scratch_in_current_context() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tdt_forward_scratch) != cudaSuccess) return nullptr;
    return p;
}

}  // namespace

extern "C" int asr_tdt_forward_noalloc(const float* encoder, const float* decoder, const float* joint_W,
                                       const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                                       const int32_t* tgt_lens, const int32_t* durations, int n_dur,
                                       int max_duration, int has_zero, int B, int T, int U, int V, int d, int S,
                                       int blank_idx, float sigma, int tf32, float* loss, double* alpha,
                                       float* log_P_blank, float* log_P_y, float* log_P_dur, float* log_prob,
                                       asr_stream_t stream) {
    const size_t need = asr_tdt_workspace_bytes(B, T, U, V, n_dur, d, tf32, 0);
    if (need == 0 && B != 0) return ASR_ERR_INVALID_ARGUMENT;
    if (need > (size_t)ASR_TDT_FORWARD_NOALLOC_SCRATCH_BYTES) return ASR_ERR_SCRATCH_LIMIT;
    void* scratch = scratch_in_current_context();
    if (!scratch) return ASR_ERR_CUDA;
    return asr_tdt_forward(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations, n_dur,
                           max_duration, has_zero, B, T, U, V, d, S, blank_idx, sigma, tf32, loss, alpha,
                           log_P_blank, log_P_y, log_P_dur, log_prob, scratch,
                           (size_t)ASR_TDT_FORWARD_NOALLOC_SCRATCH_BYTES, stream);
}
