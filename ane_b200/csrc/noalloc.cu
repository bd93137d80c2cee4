// noalloc.cu -- dense_fused_i8 for callers that cannot allocate device memory.
//
// Some callers cannot allocate device memory at the moment they run
// dense_fused_i8: a host framework that has already reserved (nearly) all of
// the GPU's memory for its own pool, so a cudaMalloc would fail; a ggml-style
// backend inside graph_compute, where every buffer was planned up front and the
// backend is not supposed to allocate; and latency-critical loops, where
// cudaMalloc/cudaFree can synchronise the device.  The workspace-taking
// ane_dense_fused_i8_dev() needs either a caller buffer or a library
// allocation; ane_dense_fused_i8_noalloc_dev() needs neither: its scratch (the
// int8 copies of A and B, the two scales and the absmax partials) lives in one
// file-scope __device__ array, so the call itself allocates nothing.
//
// Limits and sharing, stated once here and in include/ane_b200.h:
//  * The array holds kNoAllocScratchBytes (40 MiB): enough for
//    ane_dense_fused_i8_workspace_size(M, N, K) up to M = N = K = 4096.  Larger
//    problems are rejected with ANE_ERR_INVALID_ARGUMENT.
//  * Every GPU that loads this part of the library keeps the 40 MiB until the
//    process exits.
//  * All calls on a device share the one array and leave their contents in it.
//    Nothing in it needs to start at zero: every byte a call reads (codes, the
//    zero K padding, scales, partials) is written earlier in the same call.
//    Calls whose kernels overlap on the GPU (different streams, or threads
//    racing on one device) race on the array; serialise them.
//  * The first call on a device looks the array's device address up with
//    cudaGetSymbolAddress (once per device, that device current).  Make that
//    first call before any stream capture.
//  * The call returns once its kernels are enqueued.  A bounded device-side
//    wait that gives up inside them is counted in a counter of this path;
//    ane_device_timeouts() reads and resets it together with the library's
//    main counter, so check it after synchronising the stream.
#include <atomic>
#include <mutex>
#include <string>

#include "ane_internal.cuh"

namespace ane_b200 {
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)40 << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int g_noalloc_timeouts;  // target of the kernels' bounded waits on this path

struct DeviceScratch {
    std::once_flag once;
    std::atomic<bool> ready{false};  // set-up done: scratch and timeouts hold device addresses
    cudaError_t err = cudaSuccess;
    void* scratch = nullptr;
    int* timeouts = nullptr;
    int sms = 0;
    int major = 0;
};
DeviceScratch g_scratch[kMaxDevices];

}  // namespace

// Bounded-wait failures of kernels launched by the allocation-free entry point
// on the current device since the last read, and resets the count (0 if that
// entry point never ran on this device).  ane_device_timeouts() adds this to the
// library's main counter, so one call reports every timed-out wait.
int noalloc_read_and_reset_timeouts(cudaStream_t s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return 0;
    }
    DeviceScratch& d = g_scratch[dev];
    if (!d.ready.load(std::memory_order_acquire) || !d.timeouts) return 0;
    int v = 0;
    if (cudaMemcpyAsync(&v, d.timeouts, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaStreamSynchronize(s);
    if (v) cudaMemsetAsync(d.timeouts, 0, sizeof(int), s);
    return v;
}

}  // namespace ane_b200

using namespace ane_b200;

extern "C" int ane_dense_fused_i8_noalloc_dev(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu,
                                              const float* A, const float* B, float* C, void* stream) {
    const size_t need = ane_dense_fused_i8_workspace_size(M, N, K);
    if (need > kNoAllocScratchBytes) {
        set_status(ANE_ERR_INVALID_ARGUMENT,
                   "dense_fused_i8_noalloc: needs " + std::to_string(need) + " bytes of scratch, the fixed buffer holds " +
                       std::to_string(kNoAllocScratchBytes) + " (use ane_dense_fused_i8_dev with a workspace)");
        return ANE_ERR_INVALID_ARGUMENT;
    }
    if (M == 0 || N == 0) return ok();
    if (!C || (K != 0 && (!A || !B))) {
        set_status(ANE_ERR_INVALID_ARGUMENT, "dense_fused_i8_noalloc: NULL pointer");
        return ANE_ERR_INVALID_ARGUMENT;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        set_status(ANE_ERR_NO_DEVICE, "dense_fused_i8_noalloc: no usable CUDA device");
        return ANE_ERR_NO_DEVICE;
    }
    DeviceScratch& d = g_scratch[dev];
    std::call_once(d.once, [&d, dev] {
        // once per device, with that device current (it is: cudaGetDevice above)
        d.err = cudaGetSymbolAddress(&d.scratch, g_noalloc_scratch);
        if (d.err == cudaSuccess) d.err = cudaGetSymbolAddress((void**)&d.timeouts, g_noalloc_timeouts);
        if (d.err == cudaSuccess) d.err = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        if (d.err == cudaSuccess) d.err = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
        if (d.err == cudaSuccess) d.ready.store(true, std::memory_order_release);
    });
    if (d.err != cudaSuccess || !d.scratch) {
        set_status(ANE_ERR_CUDA, std::string("dense_fused_i8_noalloc: scratch set-up failed: ") + cudaGetErrorString(d.err));
        return ANE_ERR_CUDA;
    }
    if (d.major != 10) {
        set_status(ANE_ERR_NO_DEVICE, "dense_fused_i8_noalloc: needs an sm_100 (B200) device");
        return ANE_ERR_NO_DEVICE;
    }
    // Route the launchers' SM count and wait-timeout flag to this path's own
    // values so nothing lazily allocates per-device state during the call.
    const LaunchOverride ov{d.sms, d.timeouts};
    ScopedLaunchOverride guard(&ov);
    const int rc = dense_fused_on_stream(M, N, K, scale, relu, A, B, C, d.scratch, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}
