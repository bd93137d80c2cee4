// q8_0_gemv_q8.cu -- Q8_0 matvec with a Q8_0-quantized activation ("mode Q").
//
// The reference's q8_0_gemv keeps the activation in fp32
// (src/bytecode_interpreter.s:7016-7063, reproduced bit-exactly in
// q8_0_gemv.cu).  The ggml/llama.cpp convention for Q8_0 x Q8_0 instead
// quantizes the activation per 32-block to Q8_0 as well and reduces each block
// with integer dot products.  This file implements that variant:
//   quantize:  per block amax = max|x| (sequential compare, ggml's MAX), d = amax/127
//              stored as fp16(d), q = roundf(x * (d ? 1/d : 0))  (x * id is one RN multiply)
//   dot:       sumi_b = sum_j qw[j]*qx[j] (exact int32 via dp4a),
//              out[m] = sum_b float(sumi_b) * (dw_b * dx_b)
// The int32 block dots are exact; the fp32 sum over blocks runs per lane in
// block order and then across 16 lanes by xor shuffles (an order of its own,
// checked against the sequential CPU restatement within a tolerance).
//
// Memory: the weights stream through the same TMA ring as the fp32-activation
// kernel (q8_stream.cuh); the activation blocks arrive in shared memory by one
// bulk copy and are re-laid-out once per CTA as an aligned int8 array + fp32
// scales, so each dp4a operand is one aligned 32-bit load.
#include <cuda_fp16.h>

#include "ane_internal.cuh"
#include "q8_mmq.cuh"
#include "q8_stream.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {


// One warp per 32 blocks of x: thread j quantizes block (warp*32 + j)... one
// thread per block keeps ggml's sequential amax (NaN behaviour included).
__global__ void quantize_q8_0_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, uint32_t nblocks) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float* xb = x + (size_t)b * 32;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(xb + j);
        v[j] = t.x;
        v[j + 1] = t.y;
        v[j + 2] = t.z;
        v[j + 3] = t.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; j++) {
        const float a = fabsf(v[j]);
        amax = amax > a ? amax : a;
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    // a block starts at an even byte offset: write it as 17 little-endian 16-bit words
    unsigned short* blk = reinterpret_cast<unsigned short*>(out + (size_t)b * 34);
    blk[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const uint32_t lo = (uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j], id));
        const uint32_t hi = (uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j + 1], id));
        blk[1 + j / 2] = (unsigned short)(lo | (hi << 8));
    }
}

// Work split, ring and launch: q8_stream.cuh.  A compute warp owns 4 rows; lane
// = 4*pp + r takes block pair pp (blocks 2pp, 2pp+1 of the chunk) of row r.  A
// pair is 68 bytes, so it starts 4-byte aligned in the stage and is read as 17
// aligned words: the odd block's codes are words 9..16, the even block's codes
// straddle words 0..8 (one funnel shift per word).  Per lane the block terms
// are summed in block order, then across the 8 pairs by xor shuffles 4, 8, 16.
// Bytes of the activation as it arrives in shared memory: Q8_0 blocks, or fp32
// when the kernel quantizes the activation itself (XF32).
__host__ __device__ constexpr uint32_t x_raw_bytes(bool xf32, uint32_t K) { return xf32 ? K * 4 : K / 32 * 34; }

// Tagged words: one 64-bit access each (value low, tag high), so a reader never
// sees a half-written word, even from a peer GPU over NVLink.
__device__ __forceinline__ uint64_t ld_tagged(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_tagged(uint64_t* p, float value, uint32_t tag) {
    const uint64_t w = (uint64_t)__float_as_uint(value) | ((uint64_t)tag << 32);
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint4 ld_tagged2(const uint64_t* p) {
    uint64_t a, b;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
    return make_uint4((uint32_t)a, (uint32_t)(a >> 32), (uint32_t)b, (uint32_t)(b >> 32));
}
// Bounded wait until *p carries `tag`; returns the word's value (or false on timeout).
__device__ bool wait_tagged(const uint64_t* p, uint32_t tag, float* value, int* err) {
    uint64_t w = ld_tagged(p);
    if ((uint32_t)(w >> 32) != tag) {
        const long long t0 = clock64();
        while (true) {
            __nanosleep(32);
            w = ld_tagged(p);
            if ((uint32_t)(w >> 32) == tag) break;
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);
                return false;
            }
        }
    }
    *value = __uint_as_float((uint32_t)w);
    return true;
}

// XF32 = false: xq holds K/32 Q8_0 blocks.  XF32 = true: xq holds fp32 x[K] and
// every CTA quantizes it with the ggml rule (the quantize_q8_0_kernel
// arithmetic above, block by block) into the same shared-memory codes + scales,
// so the result equals quantize_q8_0 followed by the XF32 = false kernel.
// GATHER (with XF32): one projection of a row-sharded chain (Q8ChainGather,
// tagged vectors): the compute warps fill x themselves -- from the previous
// projection's tagged vector, or the fp32 input -- after the guard words of the
// previous projection carry its tag, and the rows go to every rank's vector as
// tagged words.  The producer streams weights only, so the weight tiles of the
// first ring stages load while the compute warps wait for their input.
template <bool XF32, bool GATHER>
__global__ void __launch_bounds__(32 * (kQ8MaxWarps + 1)) q8_0_gemv_q8_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ xq,
                                    float* __restrict__ out, int32_t* __restrict__ block_dots, uint32_t M, uint32_t K,
                                    uint32_t groups, uint32_t nw, uint32_t nslots, uint32_t flags, int* err,
                                    const __grid_constant__ Q8ChainGather pg) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nb = K / 32, nchunks = (nb + kQ8ChunkBlocks - 1) / kQ8ChunkBlocks;
    const uint32_t slot_bytes = nw * kQ8WarpTileBytes;
    const uint32_t xbytes = x_raw_bytes(XF32, K);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // nslots
    uint64_t* empty = full + nslots;                     // nslots
    uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + 128);
    uint8_t* xraw = smem + 256;                                                // the activation as in HBM
    float* xd = reinterpret_cast<float*>(xraw + round_up(xbytes, 128));        // nb scales
    int8_t* xs = reinterpret_cast<int8_t*>(xraw + round_up(xbytes, 128) + round_up(nb * 4, 128));  // K codes
    uint8_t* ring = reinterpret_cast<uint8_t*>(xs) + round_up(K, 128);
    const uint32_t g0 = (uint32_t)((uint64_t)groups * blockIdx.x / gridDim.x);
    const uint32_t g1 = (uint32_t)((uint64_t)groups * (blockIdx.x + 1) / gridDim.x);
    const uint32_t npass = (g1 - g0 + nw - 1) / nw, ntiles = npass * nchunks;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nslots; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], nw);
        }
        ptx::mbar_init(xbar, 1);
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    ptx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            ptx::prefetch_tmap(&wmap);
            auto issue_weights = [&](uint32_t t, uint32_t slot) {
                const uint32_t pass = t / nchunks, c = t - pass * nchunks;
                const uint32_t gp = g0 + pass * nw, nwp = min(nw, g1 - gp);
                uint8_t* dst = ring + (size_t)slot * slot_bytes;
                ptx::mbar_arrive_expect_tx(&full[slot], nwp * kQ8WarpTileBytes);
                for (uint32_t w = 0; w < nwp; w++)
                    ptx::tma_load_2d(dst + w * kQ8WarpTileBytes, &wmap, &full[slot], (int)(c * (kQ8ChunkBytes / 4)),
                                     (int)((gp + w) * kQ8RowsPerWarp));
            };
            // static weights: the first stages' weight tiles are requested before
            // the previous kernel on the stream has finished
            const uint32_t pre = (flags & ANE_Q8_WEIGHTS_STATIC) ? min(nslots, ntiles) : 0;
            for (uint32_t t = 0; t < pre; t++) issue_weights(t, t);
            ptx::griddep_wait();  // xq may be written by the previous kernel
            if constexpr (!GATHER) {  // (with GATHER the compute warps fill x)
                ptx::mbar_arrive_expect_tx(xbar, xbytes);
                ptx::bulk_load(xraw, xq, xbytes, xbar);
            }
            for (uint32_t t = pre; t < ntiles; t++) {
                const uint32_t slot = t % nslots;
                if (!ptx::mbar_wait(&empty[slot], ((t / nslots) & 1) ^ 1, err)) break;
                issue_weights(t, slot);
            }
        }
        return;
    }
    // ------------------------------------------------------------ compute
    // the token count: only the token-end kernel writes it, which precedes
    // projection 0 of a token, so later projections read it before the wait
    uint32_t tok_early = 0;
    if constexpr (GATHER) {
        if (pg.j != 0) tok_early = *reinterpret_cast<const volatile uint32_t*>(pg.tok);
    }
    ptx::griddep_wait();  // out / block_dots may belong to the previous kernel
    const uint32_t cw = warp - 1;
    uint32_t tag_out = 0;
    bool alive = true;
    if constexpr (GATHER) {
        // Every compute thread takes a share of the guard words and of x's word
        // pairs; one round issues kXU loads per thread back to back, then checks
        // their tags, and polls (bounded) only the words not there yet.
        // Cross-GPU waits only: the previous kernel on this GPU has finished.
        const uint32_t tokv = pg.j != 0 ? tok_early : *reinterpret_cast<const volatile uint32_t*>(pg.tok);
        const uint32_t tag_in = tokv * pg.nproj + pg.j;
        tag_out = tag_in + 1u;
        const uint32_t tid = cw * 32 + lane, nthr = nw * 32;
        const uint32_t nguard = pg.world * pg.prev_ctas;
        const uint32_t npairs = pg.x_from_prev ? K / 2 : 0;
        float* xf = reinterpret_cast<float*>(xraw);
        bool ok = true;
        float v;
        constexpr uint32_t kXU = 8;
        for (uint32_t base = tid; base < nguard + npairs && ok; base += nthr * kXU) {
            uint4 w[kXU];
#pragma unroll
            for (uint32_t u = 0; u < kXU; u++) {
                const uint32_t i = base + u * nthr;
                if (i < nguard) {
                    const uint32_t r = i / pg.prev_ctas, c = i - r * pg.prev_ctas;
                    const uint32_t g = (uint32_t)((uint64_t)pg.prev_groups * c / pg.prev_ctas);
                    const uint64_t* p = pg.prev + (size_t)r * pg.prev_rows + g * kQ8RowsPerWarp;
                    const uint64_t gw = ld_tagged(p);
                    w[u] = make_uint4((uint32_t)gw, (uint32_t)(gw >> 32), 0u, tag_in);
                } else if (i < nguard + npairs) {
                    w[u] = ld_tagged2(pg.prev + 2 * (i - nguard));
                }
            }
#pragma unroll
            for (uint32_t u = 0; u < kXU; u++) {
                const uint32_t i = base + u * nthr;
                if (i < nguard) {
                    if (w[u].y != tag_in) {
                        const uint32_t r = i / pg.prev_ctas, c = i - r * pg.prev_ctas;
                        const uint32_t g = (uint32_t)((uint64_t)pg.prev_groups * c / pg.prev_ctas);
                        ok = ok && wait_tagged(pg.prev + (size_t)r * pg.prev_rows + g * kQ8RowsPerWarp, tag_in, &v,
                                               err);
                    }
                } else if (i < nguard + npairs) {
                    const uint32_t pi = i - nguard;
                    if (w[u].y != tag_in) {
                        ok = ok && wait_tagged(pg.prev + 2 * pi, tag_in, &v, err);
                        w[u].x = __float_as_uint(v);
                    }
                    if (w[u].w != tag_in) {
                        ok = ok && wait_tagged(pg.prev + 2 * pi + 1, tag_in, &v, err);
                        w[u].z = __float_as_uint(v);
                    }
                    reinterpret_cast<float2*>(xf)[pi] = make_float2(__uint_as_float(w[u].x), __uint_as_float(w[u].z));
                }
            }
        }
        if (!pg.x_from_prev) {
            const float4* x4 = reinterpret_cast<const float4*>(xq);
            for (uint32_t i = tid; i < K / 4; i += nthr) reinterpret_cast<float4*>(xf)[i] = x4[i];
        }
        alive = __all_sync(0xffffffffu, ok);
        ptx::named_barrier_sync(1, nw * 32);  // x complete in shared memory
    } else {
        alive = __all_sync(0xffffffffu, ptx::mbar_wait(xbar, 0, err));  // one verdict per warp
    }
    if (alive && XF32) {
        // quantize: 4 lanes per 32-element block (8 blocks per warp step), a
        // quarter of the dependent chain per lane and no 32-value array in
        // registers (the kernel then fits 32 registers, so two CTAs of up to
        // 24 warps share an SM)
        for (uint32_t b0 = cw * 8; b0 < nb; b0 += nw * 8) {
            const uint32_t b = b0 + (lane >> 2), bb = b < nb ? b : nb - 1;
            q8_quantize_quarter(reinterpret_cast<const float*>(xraw) + (size_t)bb * 32 + (lane & 3) * 8, xs, xd, bb,
                                lane & 3, b < nb);
        }
    } else if (alive) {  // activation blocks -> aligned codes + fp32 scales (compute warps only)
        for (uint32_t i = cw * 32 + lane; i < nb * 8; i += nw * 32) {
            const unsigned short* src = reinterpret_cast<const unsigned short*>(xraw + (i >> 3) * 34 + 2 + (i & 7) * 4);
            reinterpret_cast<uint32_t*>(xs)[i] = (uint32_t)src[0] | ((uint32_t)src[1] << 16);
        }
        for (uint32_t b = cw * 32 + lane; b < nb; b += nw * 32)
            xd[b] = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(xraw + b * 34)));
    }
    __syncwarp();
    ptx::named_barrier_sync(1, nw * 32);
    const uint32_t r = lane & 3, pp = lane >> 2;
    for (uint32_t pass = 0; pass < npass && alive; pass++) {
        const uint32_t gp = g0 + pass * nw;
        const uint32_t row = (gp + cw) * kQ8RowsPerWarp + r;
        const bool active = gp + cw < g1 && row < M;
        float sum = 0.f;
        for (uint32_t c = 0; c < nchunks; c++) {
            const uint32_t t = pass * nchunks + c, slot = t % nslots;
            // one verdict per warp: after a timed-out wait every lane leaves together
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&full[slot], (t / nslots) & 1, err))) { alive = false; break; }
            const uint32_t b = c * kQ8ChunkBlocks + 2 * pp;  // first block of the pair
            if (active && b < nb) {
                const uint32_t* pw = reinterpret_cast<const uint32_t*>(ring + (size_t)slot * slot_bytes +
                                                                        cw * kQ8WarpTileBytes + r * kQ8ChunkBytes +
                                                                        pp * 68);
                int32_t s0, s1;
                q8_pair(pw, xs, xd, b, s0, s1, sum);
                if (block_dots) {
                    block_dots[(size_t)row * nb + b] = s0;
                    block_dots[(size_t)row * nb + b + 1] = s1;
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[slot]);
        }
        sum = q8_row_total(sum);
        if (active && alive && pp == 0) {
            if constexpr (GATHER) {
                for (uint32_t q = 0; q < pg.world; q++) st_tagged(pg.out[q] + row, sum, tag_out);
            } else {
                out[row] = sum;
            }
        }
    }
}

// Ends a step of a row-sharded chain: waits (bounded) until every word of the
// last projection's output on this GPU (ntok token rows of `rows` words, `ld`
// apart) carries its tag (the gathered output is complete here), then counts
// the step.  Launched in plain stream order: only peers' words can still be
// missing.  Each of the grid's CTAs checks a slice (eight loads in flight per
// thread, the words not there yet read again together each round); tok[1]
// counts CTA arrivals over all steps, and the CTA that completes this step's
// count bumps tok[0].
constexpr uint32_t kEndThreads = 1024, kEndUnroll = 8, kEndMaxCtas = 32;
__global__ void __launch_bounds__(kEndThreads) q8_chain_token_end_kernel(const uint64_t* last, uint32_t rows, size_t ld,
                                                                         uint32_t ntok, uint32_t nproj, uint32_t* tok,
                                                                         int* err) {
    __shared__ uint32_t t_s;
    if (threadIdx.x == 0) t_s = *reinterpret_cast<volatile uint32_t*>(tok);
    __syncthreads();
    const uint32_t tag = t_s * nproj + nproj, n = rows * ntok;
    const uint32_t stride = gridDim.x * kEndThreads;
    for (uint32_t base = blockIdx.x * kEndThreads + threadIdx.x; base < n; base += stride * kEndUnroll) {
        uint32_t miss = 0;
#pragma unroll
        for (uint32_t u = 0; u < kEndUnroll; u++) {
            const uint32_t i = base + u * stride;
            if (i < n && (uint32_t)(ld_tagged(last + (size_t)(i / rows) * ld + i % rows) >> 32) != tag) miss |= 1u << u;
        }
        const long long t0 = miss ? clock64() : 0;
        while (miss) {
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);  // counted; the step still ends
                break;
            }
            __nanosleep(64);
#pragma unroll
            for (uint32_t u = 0; u < kEndUnroll; u++) {
                const uint32_t i = base + u * stride;
                if (((miss >> u) & 1u) &&
                    (uint32_t)(ld_tagged(last + (size_t)(i / rows) * ld + i % rows) >> 32) == tag)
                    miss &= ~(1u << u);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(tok + 1, 1u);
        if (prev + 1u == (t_s + 1u) * gridDim.x) *reinterpret_cast<volatile uint32_t*>(tok) = t_s + 1u;
    }
}

}  // namespace

// get_rows_q8_0 (0x7C; src/bytecode_interpreter.s:12355-12408): out[r][32b+j] =
// float(q_j) * float(d) of block b of table row indices[r] (one RN multiply).
// One warp per 32-element block, lane j = element j.
__global__ void get_rows_q8_0_kernel(uint32_t n_rows, uint32_t nb, const uint8_t* __restrict__ table,
                                     const uint32_t* __restrict__ indices, float* __restrict__ out) {
    const size_t w = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (w >= (size_t)n_rows * nb) return;
    const uint32_t r = (uint32_t)(w / nb), b = (uint32_t)(w % nb);
    const uint8_t* blk = table + ((size_t)indices[r] * nb + b) * 34;
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    out[(size_t)r * nb * 32 + (size_t)b * 32 + lane] = __fmul_rn((float)(int8_t)blk[2 + lane], d);
}

int launch_get_rows_q8_0(uint32_t n_rows, uint32_t dim, const uint8_t* table, const uint32_t* indices, float* out,
                         cudaStream_t s) {
    ANE_ARG_CHECK(dim % 32 == 0, "get_rows_q8_0: dim must be a multiple of 32");
    const size_t warps = (size_t)n_rows * (dim / 32);
    if (warps == 0) return ANE_OK;
    get_rows_q8_0_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(n_rows, dim / 32, table, indices, out);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_quantize_q8_0(uint32_t K, const float* x, uint8_t* out, cudaStream_t s) {
    ANE_ARG_CHECK(K % 32 == 0, "quantize_q8_0: K must be a multiple of 32");
    ANE_ARG_CHECK(((uintptr_t)x & 15) == 0, "quantize_q8_0: x must be 16-byte aligned");
    const uint32_t nb = K / 32;
    if (nb == 0) return ANE_OK;
    quantize_q8_0_kernel<<<(nb + 127) / 128, 128, 0, s>>>(x, out, nb);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

template <bool XF32>
static Q8Plan gemv_q8_plan(uint32_t M, uint32_t K) {
    const uint32_t nb = K / 32;
    // barriers (256) + the raw activation + scales + aligned codes
    const size_t fixed = 256 + round_up((size_t)x_raw_bytes(XF32, K), 128) + round_up((size_t)nb * 4, 128) +
                         round_up(K, 128);
    return plan_q8_stream(M, K, 0, fixed);
}

template <bool XF32, bool GATHER = false>
static int launch_gemv_q8(uint32_t M, uint32_t K, const uint8_t* x, const uint8_t* W, float* out, int32_t* block_dots,
                          uint32_t flags, cudaStream_t s, const Q8ChainGather* gather = nullptr) {
    if (M == 0) return ANE_OK;
    ANE_ARG_CHECK(K % 256 == 0, "q8_0_gemv_q8: K must be a multiple of 256");
    ANE_ARG_CHECK(((uintptr_t)W & 15) == 0, "q8_0_gemv_q8: W must be 16-byte aligned");
    ANE_ARG_CHECK(((uintptr_t)x & 15) == 0, "q8_0_gemv_q8: the activation must be 16-byte aligned");
    const uint32_t nb = K / 32;
    const Q8Plan p = gemv_q8_plan<XF32>(M, K);
    ANE_ARG_CHECK(p.smem <= 200 * 1024, "q8_0_gemv_q8: K too large for the shared activation buffer");
    static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
    if (int arc = set_max_dynamic_smem(q8_0_gemv_q8_kernel<XF32, GATHER>, 200 * 1024, smem_set)) return arc;
    const uint64_t row_bytes = (uint64_t)nb * 34;
    CUtensorMap wmap;
    int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                                  kQ8ChunkBytes / 4, kQ8RowsPerWarp, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    Q8ChainGather pg{};
    if (gather) pg = *gather;
    return launch_q8_stream(q8_0_gemv_q8_kernel<XF32, GATHER>, p, s, wmap, x, out, block_dots, M, K, p.groups,
                            p.warps, p.slots, flags, device_timeout_flag(), pg);
}

int launch_q8_0_gemv_q8(uint32_t M, uint32_t K, const uint8_t* xq, const uint8_t* W, float* out, int32_t* block_dots,
                        uint32_t flags, cudaStream_t s) {
    return launch_gemv_q8<false>(M, K, xq, W, out, block_dots, flags, s);
}

int launch_mul_mat_q8_0(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, int32_t* block_dots,
                        uint32_t flags, cudaStream_t s) {
    return launch_gemv_q8<true>(M, K, reinterpret_cast<const uint8_t*>(x), W, out, block_dots, flags, s);
}

uint32_t mul_mat_q8_0_ctas(uint32_t M, uint32_t K) { return M ? gemv_q8_plan<true>(M, K).ctas : 0; }

int launch_mul_mat_q8_0_gather(uint32_t M, uint32_t K, const float* x, const uint8_t* W, const Q8ChainGather& g,
                               uint32_t flags, cudaStream_t s) {
    ANE_ARG_CHECK(M > 0 && g.world >= 1 && g.world <= 8 && g.prev && g.tok && g.nproj > 0 && g.j < g.nproj,
                  "mul_mat gather: bad arguments");
    ANE_ARG_CHECK(g.prev_ctas > 0 && g.prev_groups >= g.prev_ctas && g.prev_rows > 0,
                  "mul_mat gather: bad previous-projection split");
    ANE_ARG_CHECK(g.x_from_prev || (x && ((uintptr_t)x & 15) == 0), "mul_mat gather: fp32 input must be 16-byte aligned");
    ANE_ARG_CHECK(!g.x_from_prev || K <= g.world * g.prev_rows, "mul_mat gather: x longer than the previous output");
    for (uint32_t q = 0; q < g.world; q++) ANE_ARG_CHECK(g.out[q], "mul_mat gather: NULL rank pointer");
    const float* xs = g.x_from_prev ? reinterpret_cast<const float*>(g.prev) : x;  // 16-byte aligned either way
    return launch_gemv_q8<true, true>(M, K, reinterpret_cast<const uint8_t*>(xs), W, nullptr, nullptr, flags, s, &g);
}

int launch_q8_chain_token_end(const uint64_t* last, uint32_t rows, size_t ld, uint32_t ntok, uint32_t nproj,
                              uint32_t* tok, cudaStream_t s) {
    // one grid size per chain (the arrival count assumes it): set by the words to check
    const uint32_t n = rows * ntok, per = kEndThreads * kEndUnroll;
    const uint32_t ctas = (n + per - 1) / per < kEndMaxCtas ? (n + per - 1) / per : kEndMaxCtas;
    q8_chain_token_end_kernel<<<ctas ? ctas : 1, kEndThreads, 0, s>>>(last, rows, ld, ntok, nproj, tok,
                                                                      device_timeout_flag());
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
