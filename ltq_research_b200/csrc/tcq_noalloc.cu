// Allocation-free variant of ltq_viterbi_tb: the tail-biting Viterbi with its scratch (survivor words, gain-merge
// winners, gain candidates, middle / end states) in a fixed array that the library itself carries in device memory.
//
// Who needs it: callers that cannot allocate device memory when they quantize.  An inference engine that plans all of
// its device memory once at start-up and forbids allocation while it serves, or a binding layer (cgo / JNI / N-API /
// ctypes) that is handed device pointers for the inputs and outputs but has no CUDA allocator of its own, cannot
// provide the workspace ltq_viterbi_tb asks for.  This entry point needs only the inputs and outputs.
//
// What it costs: LTQ_NOALLOC_SCRATCH_BYTES (64 MiB) of device memory on every GPU that loads this library, held until
// the process exits.  Requests whose workspace (ltq_viterbi_tb_workspace_bytes) is larger are rejected with -2.
//
// Sharing: every call on a device uses the same array.  Calls whose kernels overlap on the GPU (for example on two
// streams) race on it and produce wrong results; serialise them (one stream, or events).  The array keeps the last
// call's contents; nothing in it has to start at zero, because every word a pass reads was written earlier in the same
// pass.
//
// Set-up: the first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device
// current) and caches it for the life of the process; make that first call before any stream capture on that device.
// A process that resets the device (cudaDeviceReset) must not call this entry on it afterwards: the cached address
// would be stale.  A failed lookup returns its own cudaError_t.
#include <cuda_runtime.h>
#include <mutex>
#include "ltq_b200.h"

#define LTQ_NOALLOC_SCRATCH_BYTES (64u << 20)

static __device__ __align__(256) unsigned char g_noalloc_scratch[LTQ_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ptr[kMaxDevices];  // device address of g_noalloc_scratch per device, set once

// Device address of the scratch on the current device, looked up once per device and kept for the life of the
// process (a cudaDeviceReset of that device makes the kept address stale).  Returns the CUDA error of the lookup
// (cudaErrorInvalidDevice for a device ordinal beyond the table).
cudaError_t scratch_on_current_device(void** out)
{
    *out = nullptr;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_ptr[dev] = p;
    }
    *out = g_ptr[dev];
    return cudaSuccess;
}
}  // namespace

extern "C" size_t ltq_viterbi_tb_noalloc_capacity(void) { return LTQ_NOALLOC_SCRATCH_BYTES; }

extern "C" int ltq_viterbi_tb_noalloc(const float* x, const float* w, int w_stride, const float* tab, const float* gains,
                                      const float* tab_hi, const float* gains_hi, float* rec, int* code, int N, int T,
                                      int nu, int K, int m, const int* m_extra, int n_extra, int Gfull, int n_cand,
                                      int sub, int U_hi, int mix, int pp, int tb_passes, int tb_cand1, int tb_window,
                                      void* stream)
{
    const size_t need = ltq_viterbi_tb_workspace_bytes(N, T, Gfull, n_cand, sub, pp, tb_window, tb_cand1);
    if (need > LTQ_NOALLOC_SCRATCH_BYTES) return -2;
    void* ws = nullptr;
    const cudaError_t e = scratch_on_current_device(&ws);
    if (e != cudaSuccess) return (int)e;
    return ltq_viterbi_tb(x, w, w_stride, tab, gains, tab_hi, gains_hi, rec, code, N, T, nu, K, m, m_extra, n_extra,
                          Gfull, n_cand, sub, U_hi, mix, pp, tb_passes, tb_cand1, tb_window, ws,
                          LTQ_NOALLOC_SCRATCH_BYTES, stream);
}
