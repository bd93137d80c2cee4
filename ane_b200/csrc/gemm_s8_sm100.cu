// gemm_s8_sm100.cu -- int8 x int8 -> int32 tensor-core GEMM for B200 (sm_100a)
// with the fused fp32 epilogue of dense_fused_i8 / dense_i8.
//
// Replaces the SME2 `smopa` loop nest of the reference handler dense_i8
// (src/bytecode_interpreter.s:1978-2446).  The arithmetic contract is the
// reference's: exact int32 accumulation over K, then per element
//   y = float_rn(acc); y = y * (sa*sb); [y = y*scale | y = y + bias[n]]; fmax(...)
// with every fp32 op a separate IEEE RN operation (no FMA contraction).
//
// Structure (one persistent CTA per SM, 192 threads, warp-specialised):
//   warp 0      TMA producer: 128x128 A tile + 256x128 B tile (int8, SWIZZLE_128B)
//               per stage into a 4-stage shared-memory ring, mbarrier complete_tx.
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues
//               tcgen05.mma.cta_group::1.kind::i8 (M=128, N=256, K=32) x4 per
//               stage into a TMEM accumulator; tcgen05.commit frees the stage.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from their TMEM lane
//               quarter, fp32 epilogue, stores.  Two TMEM accumulators (2x256
//               columns) let the epilogue of tile i overlap the MMAs of tile i+1.
// No TMA multicast anywhere (this code also runs in multi-GPU jobs).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <float.h>

#include <mutex>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes = int8 elements = one 128-B swizzle row
constexpr int UMMA_K = 32;
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK;
constexpr int B_STAGE = BN * BK;
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int ACC_COLS = BN;  // int32 accumulator columns per buffer
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr int NUM_THREADS = 192;

struct Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint32_t tmem_base;
};
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + sizeof(Barriers) + 1024;

struct Params {
    uint32_t M, N, K;
    uint32_t tiles_m, tiles_n, num_kb;
    void* C;
    size_t ldc;
    GemmEpilogue ep;
    int* err;
};

__device__ __forceinline__ float epi_f32(int32_t acc, float comb, const Params& p, uint32_t n) {
    float y = __int2float_rn(acc);
    y = __fmul_rn(y, comb);
    if (p.ep.mode == kOutDenseI8) {
        y = __fadd_rn(y, p.ep.bias[n]);
        return arm_fmax(y, p.ep.relu ? 0.0f : -FLT_MAX);
    }
    y = __fmul_rn(y, p.ep.scale);
    return p.ep.relu ? arm_fmax(y, 0.0f) : y;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_s8_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sa = smem;                              // STAGES x 16 KB
    uint8_t* sb = smem + (size_t)STAGES * A_STAGE;   // STAGES x 32 KB
    Barriers* bars = reinterpret_cast<Barriers*>(smem + (size_t)STAGES * STAGE_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t num_tiles = p.tiles_m * p.tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            ptx::mbar_init(&bars->full[s], 1);
            ptx::mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            ptx::mbar_init(&bars->tmem_full[a], 1);
            ptx::mbar_init(&bars->tmem_empty[a], 4);  // one arrive per epilogue warp
        }
        ptx::fence_mbarrier_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        ptx::tmem_alloc(&bars->tmem_base, TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool alive = true;
            for (uint32_t t = blockIdx.x; t < num_tiles && alive; t += gridDim.x) {
                const int m0 = (int)((t / p.tiles_n) * BM), n0 = (int)((t % p.tiles_n) * BN);
                for (uint32_t kb = 0; kb < p.num_kb; kb++) {
                    if (!ptx::mbar_wait(&bars->empty[stage], phase ^ 1, p.err)) { alive = false; break; }
                    ptx::mbar_arrive_expect_tx(&bars->full[stage], STAGE_BYTES);
                    ptx::tma_load_2d(sa + (size_t)stage * A_STAGE, &tmap_a, &bars->full[stage], (int)(kb * BK), m0);
                    ptx::tma_load_2d(sb + (size_t)stage * B_STAGE, &tmap_b, &bars->full[stage], (int)(kb * BK), n0);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::idesc_s8s8s32(BM, BN);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool alive = true;
            for (uint32_t t = blockIdx.x; t < num_tiles && alive; t += gridDim.x) {
                if (!ptx::mbar_wait(&bars->tmem_empty[acc], acc_phase ^ 1, p.err)) break;
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
                for (uint32_t kb = 0; kb < p.num_kb; kb++) {
                    if (!ptx::mbar_wait(&bars->full[stage], phase, p.err)) { alive = false; break; }
                    ptx::tc_fence_after();
                    const uint32_t a_addr = ptx::smem_u32(sa + (size_t)stage * A_STAGE);
                    const uint32_t b_addr = ptx::smem_u32(sb + (size_t)stage * B_STAGE);
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; k++) {
                        const uint64_t ad = ptx::sdesc_kmajor_sw128(a_addr + k * UMMA_K);
                        const uint64_t bd = ptx::sdesc_kmajor_sw128(b_addr + k * UMMA_K);
                        ptx::umma_i8(d_tmem, ad, bd, idesc, (kb | k) != 0);
                    }
                    ptx::umma_commit(&bars->empty[stage]);  // frees the smem stage when done
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!alive) break;
                ptx::umma_commit(&bars->tmem_full[acc]);  // accumulator ready for the epilogue
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const uint32_t quarter = (uint32_t)(warp & 3);  // TMEM lanes this warp may access
        const uint32_t row_in_tile = quarter * 32 + lane;
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            const uint32_t m0 = (t / p.tiles_n) * BM, n0 = (t % p.tiles_n) * BN;
            if (!ptx::mbar_wait(&bars->tmem_full[acc], acc_phase, p.err)) break;
            ptx::tc_fence_after();
            float comb = 0.0f;
            if (p.ep.mode != kOutRawI32) {
                const float s0 = p.ep.scales ? p.ep.scales[0] : p.ep.sa_imm;
                const float s1 = p.ep.scales ? p.ep.scales[1] : p.ep.sb_imm;
                comb = __fmul_rn(s0, s1);
            }
            const uint32_t m = m0 + row_in_tile;
            const uint32_t taddr = tmem_base + ((quarter * 32) << 16) + acc * ACC_COLS;
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                uint32_t r[32];
                ptx::tmem_ld_32x32b_x32(taddr + c * 32, r);
                ptx::tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    // all TMEM reads of this accumulator are done: hand it back
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&bars->tmem_empty[acc]);
                }
                const uint32_t nc = n0 + c * 32;
                if (m >= p.M || nc >= p.N) continue;
                if (p.ep.mode == kOutRawI32) {
                    int32_t* out = reinterpret_cast<int32_t*>(p.C) + (size_t)m * p.ldc + nc;
                    if (nc + 32 <= p.N && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<int4*>(out + j) = make_int4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (nc + j < p.N) out[j] = (int32_t)r[j];
                    }
                } else {
                    float* out = reinterpret_cast<float*>(p.C) + (size_t)m * p.ldc + nc;
                    if (nc + 32 <= p.N && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            float4 v;
                            v.x = epi_f32((int32_t)r[j + 0], comb, p, nc + j + 0);
                            v.y = epi_f32((int32_t)r[j + 1], comb, p, nc + j + 1);
                            v.z = epi_f32((int32_t)r[j + 2], comb, p, nc + j + 2);
                            v.w = epi_f32((int32_t)r[j + 3], comb, p, nc + j + 3);
                            *reinterpret_cast<float4*>(out + j) = v;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (nc + j < p.N) out[j] = epi_f32((int32_t)r[j], comb, p, nc + j);
                    }
                }
            }
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Fills C with the epilogue of an all-zero accumulator (K == 0).
__global__ void fill_zero_k_kernel(uint32_t M, uint32_t N, void* C, size_t ldc, GemmEpilogue ep) {
    const size_t total = (size_t)M * N;
    float comb = 0.0f;
    if (ep.mode != kOutRawI32) {
        const float s0 = ep.scales ? ep.scales[0] : ep.sa_imm;
        const float s1 = ep.scales ? ep.scales[1] : ep.sb_imm;
        comb = __fmul_rn(s0, s1);
    }
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t m = (uint32_t)(i / N), n = (uint32_t)(i % N);
        if (ep.mode == kOutRawI32) {
            reinterpret_cast<int32_t*>(C)[(size_t)m * ldc + n] = 0;
            continue;
        }
        float y = __fmul_rn(0.0f, comb);
        if (ep.mode == kOutDenseI8) {
            y = arm_fmax(__fadd_rn(y, ep.bias[n]), ep.relu ? 0.0f : -FLT_MAX);
        } else {
            y = __fmul_rn(y, ep.scale);
            if (ep.relu) y = arm_fmax(y, 0.0f);
        }
        reinterpret_cast<float*>(C)[(size_t)m * ldc + n] = y;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// K-major int8 operand: `rows` x K (row stride K bytes), box = box_rows x BK.
int make_kmajor_map(CUtensorMap* map, const int8_t* base, uint32_t rows, uint32_t K, uint32_t box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        set_status(ANE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
        return ANE_ERR_CUDA;
    }
    cuuint64_t dims[2] = {K, rows};
    cuuint64_t strides[1] = {K};
    cuuint32_t box[2] = {BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_status(ANE_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
        return ANE_ERR_CUDA;
    }
    return ANE_OK;
}

}  // namespace

int launch_gemm_s8_tc(uint32_t M, uint32_t N, uint32_t K, const int8_t* Aq, const int8_t* Bt, void* C,
                      size_t ldc, const GemmEpilogue& ep, cudaStream_t s) {
    if (M == 0 || N == 0) return ANE_OK;
    if (K == 0) return launch_fill_epilogue_zero_k(M, N, C, ldc, ep, s);
    ANE_ARG_CHECK(K % 16 == 0, "gemm: K must be a multiple of 16 (TMA row stride)");
    ANE_ARG_CHECK((reinterpret_cast<uintptr_t>(Aq) & 15) == 0 && (reinterpret_cast<uintptr_t>(Bt) & 15) == 0,
                  "gemm: int8 operands must be 16-byte aligned");
    CUtensorMap ta, tb;
    int rc = make_kmajor_map(&ta, Aq, M, K, BM);
    if (rc) return rc;
    rc = make_kmajor_map(&tb, Bt, N, K, BN);
    if (rc) return rc;
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(gemm_s8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)SMEM_BYTES);
    });
    ANE_CUDA_TRY(attr_err);
    Params p;
    p.M = M;
    p.N = N;
    p.K = K;
    p.tiles_m = (M + BM - 1) / BM;
    p.tiles_n = (N + BN - 1) / BN;
    p.num_kb = (K + BK - 1) / BK;
    p.C = C;
    p.ldc = ldc;
    p.ep = ep;
    p.err = device_timeout_flag();
    const uint32_t tiles = p.tiles_m * p.tiles_n;
    const uint32_t grid = tiles < (uint32_t)num_sms() ? tiles : (uint32_t)num_sms();
    gemm_s8_tc_kernel<<<grid, NUM_THREADS, SMEM_BYTES, s>>>(ta, tb, p);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_fill_epilogue_zero_k(uint32_t M, uint32_t N, void* C, size_t ldc, const GemmEpilogue& ep,
                                cudaStream_t s) {
    const size_t total = (size_t)M * N;
    if (total == 0) return ANE_OK;
    int g = (int)ceil_div(total, 256 * 4);
    if (g > num_sms() * 4) g = num_sms() * 4;
    fill_zero_k_kernel<<<g, 256, 0, s>>>(M, N, C, ldc, ep);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
