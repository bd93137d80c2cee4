// capi.cu -- C-ABI entry points of libane_b200: status plumbing, per-thread
// streams, host-pointer staging, and the device (`*_dev`) operations.
//
// The reference's calling contract (include/ane/ane.hpp:206-220, dispatch ->
// stream_exec) is synchronous on caller-owned host memory and reentrant across
// threads (tests/test_mnist_i8.cpp:437-449 runs Hogwild workers).  Here every
// calling thread gets its own CUDA stream and its own device staging arena, so
// concurrent callers never share mutable state; device-resident buffers are
// used in place (zero copy), host buffers are copied in and out.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "ane_internal.cuh"

namespace ane_b200 {

std::atomic<uint64_t> g_launches{0};

namespace {
thread_local int t_status = ANE_OK;
thread_local std::string t_msg;

constexpr int kMaxDevices = 64;
struct DeviceInfo {
    std::once_flag once;
    int sms = 0;
    int major = 0;
    int* timeout_flag = nullptr;
};
DeviceInfo g_dev[kMaxDevices];

DeviceInfo& device_info() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) dev = 0;
    DeviceInfo& d = g_dev[dev];
    std::call_once(d.once, [&d, dev] {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess) {
            d.sms = prop.multiProcessorCount;
            d.major = prop.major;
        }
        if (cudaMalloc(&d.timeout_flag, sizeof(int)) == cudaSuccess) cudaMemset(d.timeout_flag, 0, sizeof(int));
    });
    return d;
}

// Per-thread execution context for the synchronous, host-facing entry points.
struct ThreadCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    void* arena = nullptr;
    size_t arena_bytes = 0;
    void* ws = nullptr;  // default workspace for *_dev calls given workspace == NULL
    size_t ws_bytes = 0;
};
thread_local ThreadCtx t_ctx;

int ensure_thread_ctx() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        set_status(ANE_ERR_NO_DEVICE, "no CUDA device");
        return ANE_ERR_NO_DEVICE;
    }
    if (t_ctx.device != dev) {
        // a thread that switched devices gets fresh per-device resources
        t_ctx = ThreadCtx();
        t_ctx.device = dev;
        ANE_CUDA_TRY(cudaStreamCreateWithFlags(&t_ctx.stream, cudaStreamNonBlocking));
    }
    return ANE_OK;
}

int ensure_buffer(void** buf, size_t* have, size_t need) {
    if (*have >= need) return ANE_OK;
    if (*buf) {
        cudaFree(*buf);  // synchronises the device; the arena is idle between calls anyway
        *buf = nullptr;
        *have = 0;
    }
    size_t sz = need < ((size_t)1 << 20) ? ((size_t)1 << 20) : need + need / 4;
    if (cudaMalloc(buf, sz) != cudaSuccess) {
        cudaGetLastError();
        set_status(ANE_ERR_OUT_OF_MEMORY, "cudaMalloc of " + std::to_string(sz) + " bytes failed");
        return ANE_ERR_OUT_OF_MEMORY;
    }
    *have = sz;
    return ANE_OK;
}

bool device_accessible(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// One caller buffer of a host-facing call.
struct Arg {
    const void* user;
    size_t bytes;
    bool in, out;
    void* dev = nullptr;
    bool staged = false;
};

// Resolves every argument to a device address (staging host memory through the
// thread's arena), runs `body` on the thread stream, copies outputs back, syncs.
template <class Body>
int run_staged(std::vector<Arg>& args, size_t extra_bytes, Body body) {
    int rc = ensure_thread_ctx();
    if (rc) return rc;
    size_t need = extra_bytes;
    for (auto& a : args) {
        if (a.bytes == 0 || a.user == nullptr) continue;
        if (device_accessible(a.user)) {
            a.dev = const_cast<void*>(a.user);
        } else {
            a.staged = true;
            need += round_up(a.bytes, 256);
        }
    }
    rc = ensure_buffer(&t_ctx.arena, &t_ctx.arena_bytes, need);
    if (rc) return rc;
    uint8_t* cur = static_cast<uint8_t*>(t_ctx.arena);
    void* extra = cur;
    cur += round_up(extra_bytes, 256);
    cudaStream_t s = t_ctx.stream;
    for (auto& a : args) {
        if (!a.staged) continue;
        a.dev = cur;
        cur += round_up(a.bytes, 256);
        if (a.in) ANE_CUDA_TRY(cudaMemcpyAsync(a.dev, a.user, a.bytes, cudaMemcpyHostToDevice, s));
    }
    rc = body(s, extra);
    if (rc) {
        cudaStreamSynchronize(s);
        return rc;
    }
    for (auto& a : args)
        if (a.staged && a.out) ANE_CUDA_TRY(cudaMemcpyAsync(const_cast<void*>(a.user), a.dev, a.bytes,
                                                            cudaMemcpyDeviceToHost, s));
    ANE_CUDA_TRY(cudaStreamSynchronize(s));
    int timeouts = read_and_reset_device_timeouts(s);
    if (timeouts) {
        set_status(ANE_ERR_DEVICE_TIMEOUT, "a device-side bounded wait timed out");
        return ANE_ERR_DEVICE_TIMEOUT;
    }
    return ok();
}

inline size_t a256(size_t n) { return round_up(n, 256); }

}  // namespace

size_t fused_ws_layout(uint32_t M, uint32_t N, uint32_t K, FusedWs* w, void* base) {
    const size_t K16 = round_up(K, 16);
    const size_t pcount = ane_absmax_partials_count((size_t)M * K, (size_t)K * N);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += a256(bytes);
        return o;
    };
    const size_t N16 = round_up(N, 16);
    size_t oa = take((size_t)M * K16), ob = take(K16 * N16), os = take(2 * sizeof(float)),
           op = take(pcount * sizeof(float));
    if (w && base) {
        uint8_t* b = static_cast<uint8_t*>(base);
        w->Aq = reinterpret_cast<int8_t*>(b + oa);
        w->Bq = reinterpret_cast<int8_t*>(b + ob);
        w->scales = reinterpret_cast<float*>(b + os);
        w->partials = reinterpret_cast<float*>(b + op);
    }
    return off;
}

// The quantize prologue: one cooperative kernel when the shape allows it
// (prologue_coop.cu), else three programmatic-dependent launches.  Either way
// Aq is M x K16 and Bq is B's codes in B's layout, row stride N16.
// ANE_PROLOGUE=staged forces the latter (tuning aid).
static int launch_prologue(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq,
                           int8_t* Bq, float* scales, float* partials, cudaStream_t s) {
    static const char* force = getenv("ANE_PROLOGUE");
    const bool staged = force && !strcmp(force, "staged");
    if (!staged && prologue_coop_supported(M, N, K, A, B, Aq, Bq))
        return launch_prologue_coop(M, N, K, A, B, Aq, Bq, scales, s);
    return launch_quantize_staged(M, N, K, (uint32_t)round_up(K, 16), A, B, Aq, Bq, scales, partials, s);
}

int dense_fused_on_stream(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu, const float* A,
                          const float* B, float* C, void* ws, cudaStream_t s) {
    FusedWs w{};
    fused_ws_layout(M, N, K, &w, ws);
    const uint32_t K16 = (uint32_t)round_up(K, 16);
    int rc = launch_prologue(M, N, K, A, B, w.Aq, w.Bq, w.scales, w.partials, s);
    if (rc) return rc;
    GemmEpilogue ep{kOutFusedF32, w.scales, 0.f, 0.f, scale, relu ? 1 : 0, nullptr};
    return launch_gemm_s8_tc_kn(M, N, K16, w.Aq, w.Bq, round_up(N, 16), C, N, ep, s);
}

namespace {
thread_local const LaunchOverride* t_override = nullptr;
}  // namespace
ScopedLaunchOverride::ScopedLaunchOverride(const LaunchOverride* o) : prev_(t_override) { t_override = o; }
ScopedLaunchOverride::~ScopedLaunchOverride() { t_override = prev_; }

// --------------------------------------------------------------- status API
void set_status(int code, const std::string& msg) {
    t_status = code;
    t_msg = msg;
    if (code != ANE_OK && getenv("ANE_ABORT_ON_ERROR")) {
        fprintf(stderr, "libane_b200: %s\n", msg.c_str());
        abort();
    }
}
int ok() {
    t_status = ANE_OK;
    t_msg.clear();
    return ANE_OK;
}
int num_sms() {
    if (t_override) return t_override->sms;
    int s = device_info().sms;
    return s > 0 ? s : 148;
}
int set_max_dynamic_smem_impl(const void* kernel, int bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    ANE_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t)1 << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return ANE_OK;
    ANE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit, std::memory_order_release);  // a racing second set is harmless
    return ANE_OK;
}
int require_sm100() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        set_status(ANE_ERR_NO_DEVICE, "no CUDA device visible");
        return ANE_ERR_NO_DEVICE;
    }
    if (device_info().major != 10) {
        set_status(ANE_ERR_NO_DEVICE, "libane_b200 needs an sm_100 (B200) device");
        return ANE_ERR_NO_DEVICE;
    }
    return ANE_OK;
}
int* device_timeout_flag() {
    if (t_override) return t_override->err;
    return device_info().timeout_flag;
}
int read_and_reset_device_timeouts(cudaStream_t s) {
    int* f = device_timeout_flag();
    if (!f) return 0;
    int v = 0;
    if (cudaMemcpyAsync(&v, f, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return 0;
    cudaStreamSynchronize(s);
    if (v) cudaMemsetAsync(f, 0, sizeof(int), s);
    return v;
}

}  // namespace ane_b200

using namespace ane_b200;

#define ANE_REQUIRE_GPU()                 \
    do {                                  \
        int _rc = require_sm100();        \
        if (_rc) return _rc;              \
    } while (0)

extern "C" {

int ane_last_error(void) { return t_status; }
const char* ane_last_error_string(void) { return t_msg.c_str(); }
void ane_clear_error(void) { ok(); }
const char* ane_version(void) { return "ane_b200 0.1 (sm_100a)"; }
uint64_t ane_kernel_launch_count(void) { return g_launches.load(); }
int ane_device_timeouts(void) {
    if (require_sm100()) return 0;
    return read_and_reset_device_timeouts(nullptr) + noalloc_read_and_reset_timeouts(nullptr);
}

size_t ane_absmax_partials_count(size_t count_a, size_t count_b) {
    // absmax_blocks_for() never returns more than 1024 blocks per tensor
    (void)count_a;
    (void)count_b;
    return 2 * 1024;
}

size_t ane_dense_fused_i8_workspace_size(uint32_t M, uint32_t N, uint32_t K) {
    return fused_ws_layout(M, N, K, nullptr, nullptr);
}

// ------------------------------------------------------------- device ops
int ane_dense_fused_i8_dev(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu, const float* A,
                           const float* B, float* C, void* workspace, size_t workspace_bytes, void* stream) {
    ANE_REQUIRE_GPU();
    if (M == 0 || N == 0) return ok();
    ANE_ARG_CHECK(A && B && C, "dense_fused_i8: NULL pointer");
    const size_t need = ane_dense_fused_i8_workspace_size(M, N, K);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!workspace) {
        int rc = ensure_thread_ctx();
        if (rc) return rc;
        if (t_ctx.ws_bytes < need) cudaStreamSynchronize(s);  // old workspace may be in use on s
        rc = ensure_buffer(&t_ctx.ws, &t_ctx.ws_bytes, need);
        if (rc) return rc;
        workspace = t_ctx.ws;
    } else {
        ANE_ARG_CHECK(workspace_bytes >= need, "dense_fused_i8: workspace too small");
        ANE_ARG_CHECK(((uintptr_t)workspace & 255) == 0, "dense_fused_i8: workspace must be 256-byte aligned");
    }
    int rc = dense_fused_on_stream(M, N, K, scale, relu, A, B, C, workspace, s);
    return rc ? rc : ok();
}

int ane_quantize_pair_dev(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq,
                          int8_t* Bq, float* scales, float* partials, void* stream) {
    ANE_REQUIRE_GPU();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rc = launch_prologue(M, N, K, A, B, Aq, Bq, scales, partials, s);
    return rc ? rc : ok();
}

int ane_absmax_pair_dev(const float* A, size_t count_a, const float* B, size_t count_b, float* absmax2,
                        float* partials, void* stream) {
    ANE_REQUIRE_GPU();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int pa = absmax_blocks_for(count_a), pb = absmax_blocks_for(count_b);
    int rc = launch_absmax_partials(A, count_a, B, count_b, partials, pa, pb, s);
    if (rc) return rc;
    rc = launch_reduce_partials(partials, pa, pb, absmax2, s);
    return rc ? rc : ok();
}

int ane_quantize_pair_absmax_dev(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq,
                                 int8_t* Bq, const float* absmax2, float* scales, void* stream) {
    ANE_REQUIRE_GPU();
    // absmax2 stands in for a one-entry partials list per tensor
    int rc = launch_quantize_pair(M, N, K, (uint32_t)round_up(K, 16), A, B, Aq, Bq, scales, absmax2, 1, 1,
                                  static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_gemm_s8_kn_dev(uint32_t M, uint32_t N, uint32_t K16, const int8_t* Aq, const int8_t* Bq, uint32_t ldb,
                       const float* scales, float scale, uint8_t relu, int out_mode, void* C, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(out_mode == 0 || out_mode == 1, "gemm_s8_kn: out_mode must be 0 (fp32) or 1 (int32)");
    GemmEpilogue ep{out_mode == 0 ? kOutFusedF32 : kOutRawI32, scales, 1.f, 1.f, scale, relu ? 1 : 0, nullptr};
    int rc = launch_gemm_s8_tc_kn(M, N, K16, Aq, Bq, ldb, C, N, ep, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_gemm_s8_dev(uint32_t M, uint32_t N, uint32_t K16, const int8_t* Aq, const int8_t* Bt, const float* scales,
                    float scale, uint8_t relu, int out_mode, void* C, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(out_mode == 0 || out_mode == 1, "gemm_s8: out_mode must be 0 (fp32) or 1 (int32)");
    GemmEpilogue ep{out_mode == 0 ? kOutFusedF32 : kOutRawI32, scales, 1.f, 1.f, scale, relu ? 1 : 0, nullptr};
    int rc = launch_gemm_s8_tc(M, N, K16, Aq, Bt, C, N, ep, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_quantize_fp32_i8_dev(uint32_t count, const float* src, int8_t* dst, float* scale_out, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = ensure_thread_ctx();
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t need = ane_absmax_partials_count(count, 0) * sizeof(float);
    if (t_ctx.ws_bytes < need) cudaStreamSynchronize(s);
    rc = ensure_buffer(&t_ctx.ws, &t_ctx.ws_bytes, need);
    if (rc) return rc;
    rc = launch_quantize_flat(count, src, dst, scale_out, static_cast<float*>(t_ctx.ws), absmax_blocks_for(count), s);
    return rc ? rc : ok();
}

int ane_pack_b_i8_dev(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_pack_b(K, N, src, dst, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

// dense_i8 (A signed) and dense_u8s8 (A unsigned) on device pointers.
static int dense8_dev(bool a_unsigned, uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                      const void* A, const int8_t* B_packed, const float* bias, float* C, cudaStream_t s) {
    if (M == 0 || N == 0) return ANE_OK;
    const uint32_t M16 = (uint32_t)round_up(M, 16), K64 = (uint32_t)round_up(K, 64);
    int rc = ensure_thread_ctx();
    if (rc) return rc;
    const size_t need = (size_t)N * K64;
    if (t_ctx.ws_bytes < need) cudaStreamSynchronize(s);
    rc = ensure_buffer(&t_ctx.ws, &t_ctx.ws_bytes, need > 0 ? need : 1);
    if (rc) return rc;
    int8_t* Bt = static_cast<int8_t*>(t_ctx.ws);
    rc = launch_unpack_b_to_kmajor(K64, N, B_packed, Bt, s);
    if (rc) return rc;
    GemmEpilogue ep{kOutDenseI8, nullptr, sa, sb, 1.f, (flags & 1) ? 1 : 0, bias};
    ep.a_unsigned = a_unsigned ? 1 : 0;
    return launch_gemm_s8_tc(M16, N, K64, static_cast<const int8_t*>(A), Bt, C, N, ep, s);
}

int ane_dense_i8_dev(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags, const int8_t* A,
                     const int8_t* B_packed, const float* bias, float* C, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = dense8_dev(false, M, N, K, sa, sb, flags, A, B_packed, bias, C, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_dense_u8s8_dev(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags, const uint8_t* A,
                       const int8_t* B_packed, const float* bias, float* C, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = dense8_dev(true, M, N, K, sa, sb, flags, A, B_packed, bias, C, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

// Integer CBLAS GEMMs: operands to K-major rows (transposing where the layout
// asks for it), then the tensor-core GEMM with per-operand signedness and the
// cvt * alpha epilogue.  kind: 0 igemm, 1 ugemm, 2 usgemm.
static size_t int_gemm_ws(uint32_t M, uint32_t N, uint32_t K) {
    const size_t K16 = round_up(K, 16);
    return round_up((size_t)M * K16, 256) + round_up((size_t)N * K16, 256);
}

static int int_gemm_check(uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                          uint32_t ldc, const void* A, const void* B, const float* C) {
    ANE_ARG_CHECK((flags & ~3u) == 0, "integer gemm: unknown flag bits");
    ANE_ARG_CHECK(K % 64 == 0, "integer gemm: K must be a multiple of 64");
    ANE_ARG_CHECK(lda >= ((flags & 1) ? M : K) && ldb >= ((flags & 2) ? K : N) && ldc >= N,
                  "integer gemm: leading dimension smaller than the matrix");
    ANE_ARG_CHECK(M == 0 || N == 0 || (C && (K == 0 || (A && B))), "integer gemm: NULL pointer");
    return ANE_OK;
}

static int int_gemm_on_stream(int kind, uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                              uint32_t ldb, uint32_t ldc, float alpha, float beta, const void* A, const void* B,
                              float* C, void* ws, cudaStream_t s) {
    if (M == 0 || N == 0) return ANE_OK;
    const uint32_t K16 = (uint32_t)round_up(K, 16);
    uint8_t* Akm = static_cast<uint8_t*>(ws);
    uint8_t* Bkm = Akm + round_up((size_t)M * K16, 256);
    int rc = launch_kmajor_i8(A, lda, (flags & 1) != 0, M, K, K16, Akm, s);  // transA: A is K x M
    if (rc) return rc;
    rc = launch_kmajor_i8(B, ldb, (flags & 2) == 0, N, K, K16, Bkm, s);     // B is K x N unless transB
    if (rc) return rc;
    GemmEpilogue ep{kOutIntGemm, nullptr, 1.f, 1.f, 1.f, 0, nullptr};
    ep.a_unsigned = kind != 0;
    ep.b_unsigned = kind == 1;
    ep.acc_unsigned = kind == 1;
    ep.alpha = alpha;
    ep.beta = beta;
    return launch_gemm_s8_tc(M, N, K16, reinterpret_cast<const int8_t*>(Akm), reinterpret_cast<const int8_t*>(Bkm),
                             C, ldc, ep, s);
}

int ane_cblas_int_gemm_dev(int kind, uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                           uint32_t ldc, float alpha, float beta, const void* A, const void* B, float* C,
                           void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(kind >= 0 && kind <= 2, "integer gemm: kind must be 0 (igemm), 1 (ugemm) or 2 (usgemm)");
    int rc = int_gemm_check(flags, M, N, K, lda, ldb, ldc, A, B, C);
    if (rc) return rc;
    if (M == 0 || N == 0) return ok();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = ensure_thread_ctx();
    if (rc) return rc;
    const size_t need = int_gemm_ws(M, N, K);
    if (t_ctx.ws_bytes < need) cudaStreamSynchronize(s);
    rc = ensure_buffer(&t_ctx.ws, &t_ctx.ws_bytes, need > 0 ? need : 1);
    if (rc) return rc;
    rc = int_gemm_on_stream(kind, flags, M, N, K, lda, ldb, ldc, alpha, beta, A, B, C, t_ctx.ws, s);
    return rc ? rc : ok();
}

int ane_get_rows_q8_0_dev(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out,
                          void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(n_rows == 0 || dim == 0 || (table && indices && out), "get_rows_q8_0: NULL pointer");
    int rc = launch_get_rows_q8_0(n_rows, dim, static_cast<const uint8_t*>(table), indices, out,
                                  static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

static int kquant_dev(uint32_t fmt, uint32_t M, uint32_t K, const float* in, const void* W, float* out,
                      uint32_t flags, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(M == 0 || (in && W && out), "k-quant gemv: NULL pointer");
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "k-quant gemv: unknown flag bits");
    int rc = launch_kquant_gemv(fmt, M, K, in, static_cast<const uint8_t*>(W), out, flags,
                                static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}
int ane_kquant_gemv_ex_dev(uint8_t op, uint32_t M, uint32_t K, const float* in, const void* W, float* out,
                           uint32_t flags, void* stream) {
    ANE_ARG_CHECK(op >= 0x75 && op <= 0x79, "k-quant gemv: op must be one of 0x75-0x79");
    return kquant_dev(op - 0x75u, M, K, in, W, out, flags, stream);
}
int ane_q4_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream) {
    return kquant_dev(0, M, K, in, W, out, 0, stream);
}
int ane_q2_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream) {
    return kquant_dev(1, M, K, in, W, out, 0, stream);
}
int ane_q3_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream) {
    return kquant_dev(2, M, K, in, W, out, 0, stream);
}
int ane_q5_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream) {
    return kquant_dev(3, M, K, in, W, out, 0, stream);
}
int ane_q6_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream) {
    return kquant_dev(4, M, K, in, W, out, 0, stream);
}

int ane_get_rows_q4_0_dev(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out,
                          void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(n_rows == 0 || dim == 0 || (table && indices && out), "get_rows_q4_0: NULL pointer");
    int rc = launch_get_rows_q4_0(n_rows, dim, static_cast<const uint8_t*>(table), indices, out,
                                  static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_q4_0_gemv_ex_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, uint32_t flags,
                         void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "q4_0_gemv: unknown flag bits");
    int rc = launch_q4_0_gemv(M, K, in, static_cast<const uint8_t*>(W), out, flags, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_q4_0_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream) {
    return ane_q4_0_gemv_ex_dev(M, K, in, W, out, 0, stream);
}

int ane_q8_0_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream) {
    return ane_q8_0_gemv_ex_dev(M, K, in, W, out, 0, stream);
}

int ane_q8_0_gemv_ex_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, uint32_t flags,
                         void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "q8_0_gemv: unknown flag bits");
    int rc = launch_q8_0_gemv(M, K, in, static_cast<const uint8_t*>(W), out, flags, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_quantize_q8_0_dev(uint32_t K, const float* x, void* xq_blocks, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_quantize_q8_0(K, x, static_cast<uint8_t*>(xq_blocks), static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_q8_0_gemv_q8_dev(uint32_t M, uint32_t K, const void* xq_blocks, const void* W, float* out,
                         int32_t* block_dots, void* stream) {
    return ane_q8_0_gemv_q8_ex_dev(M, K, xq_blocks, W, out, block_dots, 0, stream);
}

int ane_q8_0_gemv_q8_ex_dev(uint32_t M, uint32_t K, const void* xq_blocks, const void* W, float* out,
                            int32_t* block_dots, uint32_t flags, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "q8_0_gemv_q8: unknown flag bits");
    int rc = launch_q8_0_gemv_q8(M, K, static_cast<const uint8_t*>(xq_blocks), static_cast<const uint8_t*>(W), out,
                                 block_dots, flags, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_mul_mat_q8_0_dev(uint32_t M, uint32_t K, const float* x, const void* W, float* out, int32_t* block_dots,
                         uint32_t flags, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "mul_mat_q8_0: unknown flag bits");
    int rc = launch_mul_mat_q8_0(M, K, x, static_cast<const uint8_t*>(W), out, block_dots, flags,
                                 static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

uint32_t ane_mul_mat_q8_0_ctas(uint32_t rows_local, uint32_t K) {
    if (require_sm100()) return 0;
    return mul_mat_q8_0_ctas(rows_local, K);
}

int ane_mul_mat_q8_0_gather_dev(uint32_t rows_local, uint32_t K, const float* x, const void* W, uint32_t world,
                                void* const* out_ranks, const void* prev, uint32_t x_from_prev, uint32_t prev_rows,
                                uint32_t prev_ctas, const uint32_t* tok, uint32_t nproj, uint32_t j, uint32_t flags,
                                void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "mul_mat_q8_0_gather: unknown flag bits");
    ANE_ARG_CHECK(world >= 1 && world <= 8 && out_ranks, "mul_mat_q8_0_gather: world must be 1..8");
    Q8ChainGather g{};
    g.world = world;
    for (uint32_t q = 0; q < world; q++) g.out[q] = static_cast<uint64_t*>(out_ranks[q]);
    g.prev = static_cast<const uint64_t*>(prev);
    g.x_from_prev = x_from_prev ? 1u : 0u;
    g.prev_rows = prev_rows;
    g.prev_groups = (prev_rows + 3) / 4;
    g.prev_ctas = prev_ctas;
    g.tok = tok;
    g.nproj = nproj;
    g.j = j;
    int rc = launch_mul_mat_q8_0_gather(rows_local, K, x, static_cast<const uint8_t*>(W), g, flags,
                                        static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_q8_0_gemv_gather_dev(uint32_t rows_local, uint32_t K, const float* x, float* xbuf, const void* W,
                             uint32_t world, void* const* out_ranks, const void* prev, uint32_t x_from_prev,
                             uint32_t prev_rows, const uint32_t* tok, uint32_t nproj, uint32_t j, uint32_t flags,
                             void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "q8_0_gemv_gather: unknown flag bits");
    ANE_ARG_CHECK(world >= 1 && world <= 8 && out_ranks, "q8_0_gemv_gather: world must be 1..8");
    ANE_ARG_CHECK(!x_from_prev || xbuf, "q8_0_gemv_gather: a chained input needs xbuf");
    Q8ChainGather g{};
    g.world = world;
    for (uint32_t q = 0; q < world; q++) {
        ANE_ARG_CHECK(out_ranks[q] && ((uintptr_t)out_ranks[q] & 7) == 0,
                      "q8_0_gemv_gather: 8-byte-aligned output pointer per rank");
        g.out[q] = static_cast<uint64_t*>(out_ranks[q]);
    }
    g.prev = static_cast<const uint64_t*>(prev);
    g.x_from_prev = x_from_prev ? 1u : 0u;
    g.prev_rows = prev_rows;
    g.tok = tok;
    g.nproj = nproj;
    g.j = j;
    int rc = launch_q8_0_gemv_gather(rows_local, K, x, xbuf, static_cast<const uint8_t*>(W), g, flags,
                                     static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_q8_chain_token_end_dev(const void* last, uint32_t len, uint32_t nproj, uint32_t* tok, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(last && tok && nproj > 0, "q8_chain_token_end: bad arguments");
    int rc = launch_q8_chain_token_end(static_cast<const uint64_t*>(last), len, len, 1, nproj, tok,
                                       static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_mul_mat_q8_0_batch_gather_dev(uint32_t rows_local, uint32_t K, uint32_t NT, const float* x, size_t ldx,
                                      const void* W, void* workspace, uint32_t world, void* const* out_ranks,
                                      size_t ldw, const void* prev, uint32_t x_from_prev, uint32_t prev_rows,
                                      const uint32_t* tok, uint32_t nproj, uint32_t j, uint32_t flags, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "mul_mat_q8_0_batch_gather: unknown flag bits");
    ANE_ARG_CHECK(world >= 1 && world <= 8 && out_ranks, "mul_mat_q8_0_batch_gather: world must be 1..8");
    ANE_ARG_CHECK(prev && tok && nproj > 0 && j < nproj && prev_rows > 0, "mul_mat_q8_0_batch_gather: bad chain");
    ANE_ARG_CHECK(ldw >= (size_t)rows_local * world && ldw >= K && (ldw % 2) == 0 && ((uintptr_t)prev & 15) == 0,
                  "mul_mat_q8_0_batch_gather: ldw must hold every rank's rows and K, be even, prev 16-byte aligned");
    Q8BatchGather g{};
    g.world = world;
    for (uint32_t q = 0; q < world; q++) {
        ANE_ARG_CHECK(out_ranks[q] && ((uintptr_t)out_ranks[q] & 7) == 0,
                      "mul_mat_q8_0_batch_gather: 8-byte-aligned output pointer per rank");
        g.out[q] = static_cast<uint64_t*>(out_ranks[q]);
    }
    g.ldw = ldw;
    g.prev = static_cast<const uint64_t*>(prev);
    g.x_from_prev = x_from_prev ? 1u : 0u;
    g.prev_rows = prev_rows;
    g.tok = tok;
    g.nproj = nproj;
    g.j = j;
    int rc = launch_mul_mat_q8_0_batch_gather(rows_local, K, NT, x, ldx, static_cast<const uint8_t*>(W), workspace,
                                              g, flags, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_q8_batch_step_end_dev(const void* last, uint32_t rows, size_t ld, uint32_t ntok, uint32_t nproj,
                              uint32_t* tok, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(last && tok && nproj > 0 && ld >= rows, "q8_batch_step_end: bad arguments");
    int rc = launch_q8_chain_token_end(static_cast<const uint64_t*>(last), rows, ld, ntok, nproj, tok,
                                       static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

size_t ane_mul_mat_q8_0_batch_workspace_size(uint32_t M, uint32_t K) {
    return mul_mat_q8_0_batch_workspace_size(M, K);
}

int ane_mul_mat_q8_0_batch_dev(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx, const void* W,
                               float* y, size_t ldy, void* workspace, uint32_t flags, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK((flags & ~ANE_Q8_WEIGHTS_STATIC) == 0, "mul_mat_q8_0_batch: unknown flag bits");
    int rc = launch_mul_mat_q8_0_batch(M, K, NT, x, ldx, static_cast<const uint8_t*>(W), y, ldy, workspace, flags,
                                       static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_quantize_pair_xrank_dev(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq,
                                int8_t* Bq, float* scales, float* partials, uint32_t world, uint32_t rank,
                                void* const* slot_peer, const void* slots, uint32_t* ctl, void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(world >= 1 && world <= 8 && rank < world, "quantize xrank: world must be 1..8, rank < world");
    ANE_ARG_CHECK(prologue_coop_supported(M, N, K, A, B, Aq, Bq),
                  "quantize xrank: needs K % 16 == 0, N % 16 == 0, 16-byte alignment and M*K + K*N >= 2^22");
    ANE_ARG_CHECK(world == 1 || (slot_peer && slots && ctl), "quantize xrank: NULL exchange pointer");
    CoopXRank x{};
    x.world = world;
    x.rank = rank;
    for (uint32_t q = 0; q < world && world > 1; q++) x.slot_peer[q] = slot_peer[q];
    x.slots = slots;
    x.ctl = ctl;
    (void)partials;  // the cooperative prologue reduces through its own control block
    int rc = launch_prologue_coop(M, N, K, A, B, Aq, Bq, scales, static_cast<cudaStream_t>(stream), &x);
    return rc ? rc : ok();
}

int ane_gemm_s8_gather_dev(uint32_t M, uint32_t N, uint32_t K16, const int8_t* Aq, const int8_t* Bq,
                           const float* scales, float scale, uint8_t relu, uint32_t world, uint32_t rank,
                           void* const* C_ranks, uint32_t ldc, uint32_t* const* ctr_ranks, uint32_t* epoch,
                           void* stream) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(world >= 2 && world <= 8 && rank < world, "gemm gather: world must be 2..8, rank < world");
    ANE_ARG_CHECK(C_ranks && ctr_ranks && epoch && scales, "gemm gather: NULL argument");
    ANE_ARG_CHECK(M > 0 && N > 0 && K16 > 0, "gemm gather: empty problem");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GatherArgs g{};
    g.world = world;
    for (uint32_t q = 0; q < world; q++) {
        g.C_rank[q] = C_ranks[q];
        g.ctr_rank[q] = ctr_ranks[q];
    }
    GemmEpilogue ep{kOutFusedF32, scales, 0.f, 0.f, scale, relu ? 1 : 0, nullptr};
    uint32_t grid = 0;
    int rc = launch_gemm_s8_tc_kn(M, N, K16, Aq, Bq, round_up(N, 16), C_ranks[rank], ldc, ep, s, &g, &grid);
    if (rc) return rc;
    rc = launch_gather_wait(ctr_ranks[rank], epoch, world * grid, s);
    return rc ? rc : ok();
}

int ane_q8_stack_plan_create(const ane_q8_stack_proj* projs, uint32_t nproj, uint32_t world, uint32_t rank,
                             uint32_t* ctl, void** plan) {
    ANE_REQUIRE_GPU();
    int rc = stack_plan_create(projs, nproj, world, rank, ctl, plan);
    return rc ? rc : ok();
}

int ane_q8_stack_run(void* plan, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = stack_plan_run(plan, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

void ane_q8_stack_plan_free(void* plan) { stack_plan_free(plan); }

namespace {
// cuMemGetAddressRange through the runtime's driver entry point (no -lcuda).
using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
MemGetAddressRangeFn address_range_fn() {
    static MemGetAddressRangeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (MemGetAddressRangeFn) nullptr;
        return reinterpret_cast<MemGetAddressRangeFn>(f);
    }();
    return fn;
}
}  // namespace

extern "C++" {
namespace ane_b200 {
size_t device_bytes_from(const void* p) {
    auto fn = address_range_fn();
    if (!fn || !p) return 0;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, (CUdeviceptr)p) != CUDA_SUCCESS) {
        cudaGetLastError();
        return 0;
    }
    return (size_t)(base + size - (CUdeviceptr)p);
}
}  // namespace ane_b200
}

int ane_ipc_get_handle(const void* dev_ptr, void* handle64, uint64_t* offset) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(dev_ptr && handle64 && offset, "ipc: NULL argument");
    auto fn = address_range_fn();
    if (!fn) {
        set_status(ANE_ERR_CUDA, "ipc: cuMemGetAddressRange unavailable");
        return ANE_ERR_CUDA;
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS) {
        set_status(ANE_ERR_INVALID_ARGUMENT, "ipc: pointer is not device memory");
        return ANE_ERR_INVALID_ARGUMENT;
    }
    cudaIpcMemHandle_t h;
    ANE_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(handle64, &h, sizeof(h));
    *offset = (uint64_t)((CUdeviceptr)dev_ptr - base);
    return ok();
}

int ane_ipc_open_handle(const void* handle64, void** base) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(handle64 && base, "ipc: NULL argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    ANE_CUDA_TRY(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
    return ok();
}

int ane_ipc_close_handle(void* base) {
    ANE_REQUIRE_GPU();
    ANE_CUDA_TRY(cudaIpcCloseMemHandle(base));
    return ok();
}

// ------------------------------------------------- host-facing (synchronous)
int ane_quantize_fp32_i8(uint32_t count, const float* src, int8_t* dst, float* scale_out) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(scale_out != nullptr, "quantize_fp32_i8: NULL scale_out");
    ANE_ARG_CHECK(count == 0 || (src && dst), "quantize_fp32_i8: NULL pointer");
    std::vector<Arg> args = {{src, (size_t)count * 4, true, false},
                             {dst, (size_t)count, false, true},
                             {scale_out, 4, false, true}};
    const size_t pbytes = ane_absmax_partials_count(count, 0) * sizeof(float);
    return run_staged(args, pbytes, [&](cudaStream_t s, void* extra) {
        return launch_quantize_flat(count, (const float*)args[0].dev, (int8_t*)args[1].dev, (float*)args[2].dev,
                                    (float*)extra, absmax_blocks_for(count), s);
    });
}

int ane_dequantize_i8_fp32(uint32_t count, float scale, const int8_t* src, float* dst) {
    ANE_REQUIRE_GPU();
    if (count == 0) return ok();
    ANE_ARG_CHECK(src && dst, "dequantize_i8_fp32: NULL pointer");
    std::vector<Arg> args = {{src, (size_t)count, true, false}, {dst, (size_t)count * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_dequantize(count, scale, (const int8_t*)args[0].dev, (float*)args[1].dev, s);
    });
}

int ane_pack_b_i8(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst) {
    ANE_REQUIRE_GPU();
    const size_t out_bytes = (size_t)((N + 15) / 16) * ((K + 3) / 4) * 64;
    if (out_bytes == 0) return ok();
    ANE_ARG_CHECK(dst && (src || (size_t)K * N == 0), "pack_b_i8: NULL pointer");
    std::vector<Arg> args = {{src, (size_t)K * N, true, false}, {dst, out_bytes, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_pack_b(K, N, (const int8_t*)args[0].dev, (int8_t*)args[1].dev, s);
    });
}

int ane_quantize_fp32_i8_channelwise(uint32_t rows, uint32_t cols, const float* src, int8_t* dst, float* scales) {
    ANE_REQUIRE_GPU();
    if (rows == 0) return ok();
    ANE_ARG_CHECK(src && dst && scales, "quantize_fp32_i8_channelwise: NULL pointer");
    std::vector<Arg> args = {{src, (size_t)rows * cols * 4, true, false},
                             {dst, (size_t)rows * cols, false, true},
                             {scales, (size_t)rows * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_quantize_channelwise(rows, cols, (const float*)args[0].dev, (int8_t*)args[1].dev,
                                           (float*)args[2].dev, s);
    });
}

// dense_i8 / dense_u8s8 on any pointer kind (the reference's synchronous contract).
static int dense8_host(bool a_unsigned, uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                       const void* A, const int8_t* B_packed, const float* bias, float* C) {
    ANE_REQUIRE_GPU();
    if (M == 0 || N == 0) return ok();
    ANE_ARG_CHECK(A && B_packed && bias && C, "dense_i8: NULL pointer");
    const size_t M16 = round_up(M, 16), K64 = round_up(K, 64);
    const size_t bp_bytes = ceil_div(N, 16) * (K64 / 4) * 64;
    std::vector<Arg> args = {{A, M16 * K64, true, false},
                             {B_packed, bp_bytes, true, false},
                             {bias, (size_t)N * 4, true, false},
                             {C, M16 * N * 4, false, true}};
    const size_t bt_bytes = (size_t)N * K64;
    return run_staged(args, bt_bytes, [&](cudaStream_t s, void* extra) {
        int8_t* Bt = static_cast<int8_t*>(extra);
        int rc = launch_unpack_b_to_kmajor((uint32_t)K64, N, (const int8_t*)args[1].dev, Bt, s);
        if (rc) return rc;
        GemmEpilogue ep{kOutDenseI8, nullptr, sa, sb, 1.f, (flags & 1) ? 1 : 0, (const float*)args[2].dev};
        ep.a_unsigned = a_unsigned ? 1 : 0;
        return launch_gemm_s8_tc((uint32_t)M16, N, (uint32_t)K64, (const int8_t*)args[0].dev, Bt, args[3].dev, N,
                                 ep, s);
    });
}

int ane_dense_i8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags, const int8_t* A,
                 const int8_t* B_packed, const float* bias, float* C) {
    return dense8_host(false, M, N, K, sa, sb, flags, A, B_packed, bias, C);
}

int ane_dense_u8s8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags, const uint8_t* A,
                   const int8_t* B_packed, const float* bias, float* C) {
    return dense8_host(true, M, N, K, sa, sb, flags, A, B_packed, bias, C);
}

static int int_gemm_host(int kind, uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                         uint32_t ldc, float alpha, float beta, const void* A, const void* B, float* C) {
    ANE_REQUIRE_GPU();
    int rc = int_gemm_check(flags, M, N, K, lda, ldb, ldc, A, B, C);
    if (rc) return rc;
    if (M == 0 || N == 0) return ok();
    // bytes each strided operand spans
    const bool ta = flags & 1, tb = flags & 2;
    const size_t a_bytes = K == 0 ? 0 : ta ? (size_t)(K - 1) * lda + M : (size_t)(M - 1) * lda + K;
    const size_t b_bytes = K == 0 ? 0 : tb ? (size_t)(N - 1) * ldb + K : (size_t)(K - 1) * ldb + N;
    const size_t c_bytes = ((size_t)(M - 1) * ldc + N) * 4;
    std::vector<Arg> args = {{A, a_bytes, true, false}, {B, b_bytes, true, false}, {C, c_bytes, true, true}};
    return run_staged(args, int_gemm_ws(M, N, K), [&](cudaStream_t s, void* extra) {
        return int_gemm_on_stream(kind, flags, M, N, K, lda, ldb, ldc, alpha, beta, args[0].dev, args[1].dev,
                                  (float*)args[2].dev, extra, s);
    });
}

int ane_cblas_igemm(uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                    float alpha, float beta, const void* A, const void* B, float* C) {
    return int_gemm_host(0, flags, M, N, K, lda, ldb, ldc, alpha, beta, A, B, C);
}
int ane_cblas_ugemm(uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                    float alpha, float beta, const void* A, const void* B, float* C) {
    return int_gemm_host(1, flags, M, N, K, lda, ldb, ldc, alpha, beta, A, B, C);
}
int ane_cblas_usgemm(uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                     float alpha, float beta, const void* A, const void* B, float* C) {
    return int_gemm_host(2, flags, M, N, K, lda, ldb, ldc, alpha, beta, A, B, C);
}

// ---- MNIST-i8 training opcodes on any pointer kind
int ane_elementwise_scaled_add_fp32(uint32_t count, float scale, const float* a, const float* b, float* out) {
    ANE_REQUIRE_GPU();
    if (count == 0) return ok();
    ANE_ARG_CHECK(a && b && out, "elementwise_scaled_add_fp32: NULL pointer");
    std::vector<Arg> args = {{a, (size_t)count * 4, true, false},
                             {b, (size_t)count * 4, true, false},
                             {out, (size_t)count * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_scaled_add_f32(count, scale, (const float*)args[0].dev, (const float*)args[1].dev,
                                     (float*)args[2].dev, s);
    });
}

int ane_relu_backward_fp32(uint32_t count, const float* act, const float* grad, float* out) {
    ANE_REQUIRE_GPU();
    if (count == 0) return ok();
    ANE_ARG_CHECK(act && grad && out, "relu_backward_fp32: NULL pointer");
    std::vector<Arg> args = {{act, (size_t)count * 4, true, false},
                             {grad, (size_t)count * 4, true, false},
                             {out, (size_t)count * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_relu_backward_f32(count, (const float*)args[0].dev, (const float*)args[1].dev,
                                        (float*)args[2].dev, s);
    });
}

int ane_transpose_fp32(uint32_t M, uint32_t N, const float* src, float* dst) {
    ANE_REQUIRE_GPU();
    if (M == 0 || N == 0) return ok();
    ANE_ARG_CHECK(src && dst, "transpose_fp32: NULL pointer");
    std::vector<Arg> args = {{src, (size_t)M * N * 4, true, false}, {dst, (size_t)M * N * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_transpose_f32(M, N, (const float*)args[0].dev, (float*)args[1].dev, s);
    });
}

int ane_count_matches(uint32_t count, const int32_t* pred, const uint8_t* labels, int32_t* out) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(out && (count == 0 || (pred && labels)), "count_matches: NULL pointer");
    std::vector<Arg> args = {{pred, (size_t)count * 4, true, false},
                             {labels, (size_t)count, true, false},
                             {out, 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_count_matches(count, (const int32_t*)args[0].dev, (const uint8_t*)args[1].dev,
                                    (int32_t*)args[2].dev, s);
    });
}

int ane_dense_fp32(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A, const float* B,
                   const float* bias, float* C) {
    ANE_REQUIRE_GPU();
    if (M == 0 || N == 0) return ok();
    ANE_ARG_CHECK(A && B && bias && C, "dense_fp32: NULL pointer");
    const size_t M16 = round_up(M, 16);
    std::vector<Arg> args = {{A, M16 * K * 4, true, false},
                             {B, (size_t)K * N * 4, true, false},
                             {bias, (size_t)N * 4, true, false},
                             {C, M16 * N * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_dense_f32(M, N, K, scale, flags, (const float*)args[0].dev, (const float*)args[1].dev,
                                (const float*)args[2].dev, (float*)args[3].dev, s);
    });
}

int ane_softmax_argmax_fp32(uint32_t batch, uint32_t cols, const float* logits, float* probs, const uint8_t* labels,
                            float* g_out, int32_t* argmax) {
    ANE_REQUIRE_GPU();
    if (batch == 0) return ok();
    ANE_ARG_CHECK(cols >= 16 && cols % 16 == 0, "softmax_argmax_fp32: cols must be a positive multiple of 16");
    ANE_ARG_CHECK(logits && probs && labels && g_out && argmax, "softmax_argmax_fp32: NULL pointer");
    const size_t bytes = (size_t)batch * cols * 4;
    // only the first 16 columns of each g_out row are written: copy it in too
    std::vector<Arg> args = {{logits, bytes, true, false},
                             {probs, bytes, false, true},
                             {labels, batch, true, false},
                             {g_out, bytes, true, true},
                             {argmax, (size_t)batch * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_softmax_argmax_f32(batch, cols, (const float*)args[0].dev, (float*)args[1].dev,
                                         (const uint8_t*)args[2].dev, (float*)args[3].dev, (int32_t*)args[4].dev, s);
    });
}

// device-pointer forms, asynchronous on `stream`
int ane_elementwise_scaled_add_fp32_dev(uint32_t count, float scale, const float* a, const float* b, float* out,
                                        void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_scaled_add_f32(count, scale, a, b, out, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}
int ane_relu_backward_fp32_dev(uint32_t count, const float* act, const float* grad, float* out, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_relu_backward_f32(count, act, grad, out, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}
int ane_transpose_fp32_dev(uint32_t M, uint32_t N, const float* src, float* dst, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_transpose_f32(M, N, src, dst, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}
int ane_count_matches_dev(uint32_t count, const int32_t* pred, const uint8_t* labels, int32_t* out, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_count_matches(count, pred, labels, out, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}
int ane_dense_fp32_dev(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A, const float* B,
                       const float* bias, float* C, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_dense_f32(M, N, K, scale, flags, A, B, bias, C, static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}
int ane_softmax_argmax_fp32_dev(uint32_t batch, uint32_t cols, const float* logits, float* probs,
                                const uint8_t* labels, float* g_out, int32_t* argmax, void* stream) {
    ANE_REQUIRE_GPU();
    int rc = launch_softmax_argmax_f32(batch, cols, logits, probs, labels, g_out, argmax,
                                       static_cast<cudaStream_t>(stream));
    return rc ? rc : ok();
}

int ane_q4_0_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    ANE_REQUIRE_GPU();
    if (M == 0) return ok();
    ANE_ARG_CHECK(K % 32 == 0, "q4_0_gemv: K must be a multiple of 32");
    ANE_ARG_CHECK(in && W && out, "q4_0_gemv: NULL pointer");
    std::vector<Arg> args = {{in, (size_t)K * 4, true, false},
                             {W, (size_t)M * (K / 32) * 18, true, false},
                             {out, (size_t)M * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_q4_0_gemv(M, K, (const float*)args[0].dev, (const uint8_t*)args[1].dev, (float*)args[2].dev, 0, s);
    });
}

static int kquant_host(uint32_t fmt, uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    ANE_REQUIRE_GPU();
    if (M == 0) return ok();
    ANE_ARG_CHECK(in && W && out, "k-quant gemv: NULL pointer");
    const size_t nsb = K / 256;
    std::vector<Arg> args = {{in, nsb > 0 ? nsb * 256 * 4 : 4, true, false},
                             {W, nsb > 0 ? (size_t)M * nsb * kquant_block_bytes(fmt) : 4, true, false},
                             {out, (size_t)M * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_kquant_gemv(fmt, M, K, (const float*)args[0].dev, (const uint8_t*)args[1].dev,
                                  (float*)args[2].dev, 0, s);
    });
}
int ane_q4_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    return kquant_host(0, M, K, in, W, out);
}
int ane_q2_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    return kquant_host(1, M, K, in, W, out);
}
int ane_q3_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    return kquant_host(2, M, K, in, W, out);
}
int ane_q5_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    return kquant_host(3, M, K, in, W, out);
}
int ane_q6_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    return kquant_host(4, M, K, in, W, out);
}

int ane_get_rows_q4_0(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(dim % 32 == 0, "get_rows_q4_0: dim must be a multiple of 32");
    if (n_rows == 0 || dim == 0) return ok();
    ANE_ARG_CHECK(table && indices && out, "get_rows_q4_0: NULL pointer");
    // the table has no size in the reference's encoding: copy rows up to the largest index
    uint32_t max_idx = 0;
    if (device_accessible(indices) && !device_accessible(table)) {
        set_status(ANE_ERR_INVALID_ARGUMENT, "get_rows_q4_0: host table with device indices");
        return ANE_ERR_INVALID_ARGUMENT;
    }
    if (!device_accessible(table))
        for (uint32_t r = 0; r < n_rows; r++) max_idx = indices[r] > max_idx ? indices[r] : max_idx;
    const size_t row_bytes = (size_t)(dim / 32) * 18;
    std::vector<Arg> args = {{table, device_accessible(table) ? 1 : ((size_t)max_idx + 1) * row_bytes, true, false},
                             {indices, (size_t)n_rows * 4, true, false},
                             {out, (size_t)n_rows * dim * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_get_rows_q4_0(n_rows, dim, (const uint8_t*)args[0].dev, (const uint32_t*)args[1].dev,
                                    (float*)args[2].dev, s);
    });
}

int ane_get_rows_q8_0(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out) {
    ANE_REQUIRE_GPU();
    ANE_ARG_CHECK(dim % 32 == 0, "get_rows_q8_0: dim must be a multiple of 32");
    if (n_rows == 0 || dim == 0) return ok();
    ANE_ARG_CHECK(table && indices && out, "get_rows_q8_0: NULL pointer");
    // the table has no size in the reference's encoding: copy rows up to the largest index
    uint32_t max_idx = 0;
    if (device_accessible(indices) && !device_accessible(table)) {
        set_status(ANE_ERR_INVALID_ARGUMENT, "get_rows_q8_0: host table with device indices");
        return ANE_ERR_INVALID_ARGUMENT;
    }
    if (!device_accessible(table))
        for (uint32_t r = 0; r < n_rows; r++) max_idx = indices[r] > max_idx ? indices[r] : max_idx;
    const size_t row_bytes = (size_t)(dim / 32) * 34;
    std::vector<Arg> args = {{table, device_accessible(table) ? 1 : ((size_t)max_idx + 1) * row_bytes, true, false},
                             {indices, (size_t)n_rows * 4, true, false},
                             {out, (size_t)n_rows * dim * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_get_rows_q8_0(n_rows, dim, (const uint8_t*)args[0].dev, (const uint32_t*)args[1].dev,
                                    (float*)args[2].dev, s);
    });
}

int ane_dense_fused_i8(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu, const float* A,
                       const float* B, float* C) {
    ANE_REQUIRE_GPU();
    if (M == 0 || N == 0) return ok();
    ANE_ARG_CHECK(C && (K == 0 || (A && B)), "dense_fused_i8: NULL pointer");
    std::vector<Arg> args = {{A, (size_t)M * K * 4, true, false},
                             {B, (size_t)K * N * 4, true, false},
                             {C, (size_t)M * N * 4, false, true}};
    const size_t ws = ane_dense_fused_i8_workspace_size(M, N, K);
    return run_staged(args, ws, [&](cudaStream_t s, void* extra) {
        return dense_fused_on_stream(M, N, K, scale, relu, (const float*)args[0].dev, (const float*)args[1].dev,
                                     (float*)args[2].dev, extra, s);
    });
}

int ane_q8_0_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out) {
    ANE_REQUIRE_GPU();
    if (M == 0) return ok();
    ANE_ARG_CHECK(K % 32 == 0, "q8_0_gemv: K must be a multiple of 32");
    ANE_ARG_CHECK(in && W && out, "q8_0_gemv: NULL pointer");
    std::vector<Arg> args = {{in, (size_t)K * 4, true, false},
                             {W, (size_t)M * (K / 32) * 34, true, false},
                             {out, (size_t)M * 4, false, true}};
    return run_staged(args, 0, [&](cudaStream_t s, void*) {
        return launch_q8_0_gemv(M, K, (const float*)args[0].dev, (const uint8_t*)args[1].dev, (float*)args[2].dev, 0, s);
    });
}

}  // extern "C"
