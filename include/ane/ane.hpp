#pragma once
/*
 * ane/ane.hpp -- drop-in C++ front end of the ane library for Linux + B200.
 *
 * Source-compatible with the reference header (joshmorgan1000/ane,
 * include/ane/ane.hpp) for the quantized dense hot path:
 *   - namespace ane, enum class Op with the reference's opcode values
 *     (ane.hpp:47-177) plus dense_fused_i8 = 0x80 (README.md:87-97);
 *   - ane::dispatch(Op, args...) packs immediates and pointers by sizeof with no
 *     padding (ane.hpp:206-220) and calls the C symbol stream_exec;
 *   - ane::program accumulates several opcodes into one stream (ane.hpp:229-352).
 * The reference version #errors off Apple aarch64 and needs <simd/simd.h>; this
 * one compiles anywhere and links against libane_b200.so, whose stream_exec
 * runs the hot-path opcodes on the GPU (see include/ane_b200.h).  Errors that
 * the reference could only express as undefined behaviour are recorded in a
 * thread-local status: ane::last_error() / ane_last_error().
 */
#include <concepts>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <new>
#include <type_traits>
#include <vector>

#include "../ane_b200.h"

namespace ane {
namespace interpreter {
// The C ABI entry point (reference: ane.hpp:37-39).  Defined in libane_b200.so.
using ::stream_exec;
}  // namespace interpreter

enum class Op : uint8_t {
    reserved_0x00 = 0x00,
    zero_za = 0x01,
    acc_smopa = 0x02,
    acc_umopa = 0x03,
    acc_usmopa = 0x04,
    acc_sumopa = 0x05,
    store_tiles = 0x06,
    smopa_2x2 = 0x07,
    umopa_2x2 = 0x08,
    usmopa_2x2 = 0x09,
    load_bias = 0x0A,
    scale_store = 0x0B,
    elementwise_add_fp32 = 0x0C,
    elementwise_scaled_add_fp32 = 0x0D,   // executed on the GPU
    elementwise_mul_fp32 = 0x0E,
    relu_backward_fp32 = 0x0F,            // executed on the GPU
    scatter_tile_fp32 = 0x10,
    transpose_fp32 = 0x11,                // executed on the GPU
    softmax_argmax_fp32 = 0x12,           // executed on the GPU
    luti4_op = 0x13,
    luti2_op = 0x14,
    dense_fp32 = 0x15,                    // executed on the GPU
    count_matches = 0x16,                 // executed on the GPU
    reduce_sum_fp32 = 0x17,
    dense_i8 = 0x18,                      // executed on the GPU
    quantize_fp32_i8 = 0x19,              // executed on the GPU
    dequantize_i8_fp32 = 0x1A,            // executed on the GPU
    pack_b_i8 = 0x1B,                     // executed on the GPU
    quantize_fp32_i8_channelwise = 0x1C,  // executed on the GPU
    transpose_i8 = 0x1D,
    dense_u8s8 = 0x1E,                    // executed on the GPU
    load = 0x1F,
    store = 0x20,
    l2_squared_fp32 = 0x21,
    l2_squared_bf16 = 0x22,
    l2_squared_f64 = 0x23,
    cosine_dist_fp32 = 0x24,
    cosine_dist_bf16 = 0x25,
    cosine_dist_f64 = 0x26,
    normalize_fp32 = 0x27,
    dct2_forward_fp32 = 0x28,
    dct2_inverse_fp32 = 0x29,
    threshold_bitmap_fp32 = 0x2A,
    welford_stats_fp32 = 0x2B,
    quantize_pack_4bit_fp32 = 0x2C,
    threshold_8bit = 0x2D,
    quantize_accum_2bit = 0x2E,
    accum_8bit = 0x2F,
    soa_sub_scale_bf16 = 0x30,
    soa_luti2_accum = 0x31,
    soa_luti4_accum = 0x32,
    bitmap_score_pipeline = 0x33,
    mov_zreg = 0x34,
    loop_begin = 0x35,
    loop_end = 0x36,
    set_param = 0x37,
    load_param = 0x38,
    store_param = 0x39,
    advance_param = 0x3A,
    fadd_zreg = 0x3B,
    fsub_zreg = 0x3C,
    fmul_zreg = 0x3D,
    fmla_zreg = 0x3E,
    and_zreg = 0x3F,
    orr_zreg = 0x40,
    eor_zreg = 0x41,
    not_zreg = 0x42,
    lsl_zreg = 0x43,
    lsr_zreg = 0x44,
    asr_zreg = 0x45,
    load_zt0 = 0x46,
    luti2_zreg = 0x47,
    luti4_zreg = 0x48,
    smopa_zreg = 0x49,
    umopa_zreg = 0x4A,
    usmopa_zreg = 0x4B,
    fmopa_zreg = 0x4C,
    cblas_sgemm = 0x4D,
    fclamp_zreg = 0x4E,
    faddv_zreg = 0x4F,
    frsqrt_zreg = 0x50,
    rms_norm_fp32 = 0x51,
    broadcast_scalar_zreg = 0x52,
    fscale_zreg = 0x53,
    silu_fp32 = 0x54,
    rope_fp32 = 0x55,
    softmax_fp32 = 0x56,
    q8_0_gemv = 0x57,  // executed on the GPU
    q4_0_gemv = 0x58,                     // executed on the GPU
    fdot_zreg = 0x59,
    fmla_wide_zreg = 0x5A,
    fadd_wide_zreg = 0x5B,
    fsub_wide_zreg = 0x5C,
    fmul_wide_zreg = 0x5D,
    load_wide_param = 0x5E,
    store_wide_param = 0x5F,
    cblas_bfgemm = 0x60,
    cblas_igemm = 0x61,                   // executed on the GPU
    cblas_ugemm = 0x62,                   // executed on the GPU
    cblas_usgemm = 0x63,                  // executed on the GPU
    gemm_tile_fp32 = 0x64,
    softmax_partial_fp32 = 0x65,
    softmax_correct_fp32 = 0x66,
    reduce_sum_sq_fp32 = 0x67,
    reduce_col_sum_fp32 = 0x68,
    silu_backward_fp32 = 0x69,
    softmax_backward_fp32 = 0x6A,
    gelu_fp32 = 0x6B,
    layer_norm_fp32 = 0x6C,
    causal_mask_fp32 = 0x6D,
    adam_step_fp32 = 0x6E,
    gelu_backward_fp32 = 0x6F,
    rms_norm_backward_fp32 = 0x70,
    layer_norm_backward_fp32 = 0x71,
    rope_backward_fp32 = 0x72,
    cross_entropy_fp32 = 0x73,
    elementwise_sub_fp32 = 0x74,
    q4_k_gemv = 0x75,                     // executed on the GPU
    q2_k_gemv = 0x76,                     // executed on the GPU
    q3_k_gemv = 0x77,                     // executed on the GPU
    q5_k_gemv = 0x78,                     // executed on the GPU
    q6_k_gemv = 0x79,                     // executed on the GPU
    flash_attention_fp32 = 0x7A,
    get_rows_fp32 = 0x7B,
    get_rows_q8_0 = 0x7C,                 // executed on the GPU
    get_rows_q4_0 = 0x7D,                 // executed on the GPU
    dense_strided_fp32 = 0x7E,
    advance_param_stride = 0x7F,
    dense_fused_i8 = 0x80,  // new: quantize(A), quantize(B), int8 GEMM, rescale, ReLU
    NUM_OPCODES = 0x81,
};

// Scalar immediates accepted by dispatch (reference tiles/concepts.hpp:18-37,
// minus Apple's bfloat16_t).
template <typename T>
concept ValidZType = std::same_as<T, float> || std::same_as<T, int32_t> || std::same_as<T, uint32_t> ||
                     std::same_as<T, int> || std::same_as<T, unsigned int> || std::same_as<T, int16_t> ||
                     std::same_as<T, uint16_t> || std::same_as<T, int8_t> || std::same_as<T, uint8_t> ||
                     std::same_as<T, char> || std::same_as<T, unsigned char> || std::same_as<T, double> ||
                     std::same_as<T, int64_t> || std::same_as<T, uint64_t> || std::same_as<T, long> ||
                     std::same_as<T, unsigned long> || std::same_as<T, long long> ||
                     std::same_as<T, unsigned long long>;

// 64-byte-aligned pointer wrapper (reference tiles/z_stream.hpp:112-119).
struct aligned_pointer {
    void* ptr;
    explicit aligned_pointer(void* p) : ptr(p) {
        if ((reinterpret_cast<uintptr_t>(ptr) & 0x3F) != 0) throw std::bad_alloc();
    }
};

template <typename T>
concept AllowedParameterTypes =
    ValidZType<T> || std::same_as<T, bool> || std::is_pointer_v<T> || std::is_same_v<T, aligned_pointer>;

// Encodes one opcode and runs it (reference ane.hpp:206-220).
template <typename... Args>
    requires(AllowedParameterTypes<Args> && ...)
inline void dispatch(Op op, Args... args) {
    constexpr size_t size_needed = 1 + (0 + ... + sizeof(Args));
    alignas(8) uint8_t bytecodes[size_needed] = {};
    bytecodes[0] = static_cast<uint8_t>(op);
    size_t offset = 1;
    auto emit = [&](auto arg) {
        std::memcpy(&bytecodes[offset], &arg, sizeof(arg));
        offset += sizeof(arg);
    };
    (emit(args), ...);
    asm volatile("" ::: "memory");
    interpreter::stream_exec(bytecodes, size_needed);
}

// Status of the calling thread's last dispatch / program::exec (0 = OK).
inline int last_error() { return ane_last_error(); }
inline const char* last_error_string() { return ane_last_error_string(); }

// Multi-opcode stream (reference ane.hpp:229-352; the SME-register helpers
// exec_into / exec_returning have no GPU meaning and are not provided).
class program {
    std::vector<uint8_t> bytecodes_;
    std::vector<size_t> loop_marks_;

public:
    template <typename... Args>
        requires(AllowedParameterTypes<Args> && ...)
    program& emit(Op op, Args... args) {
        bytecodes_.push_back(static_cast<uint8_t>(op));
        auto append_arg = [&](auto arg) {
            const auto* p = reinterpret_cast<const uint8_t*>(&arg);
            bytecodes_.insert(bytecodes_.end(), p, p + sizeof(arg));
        };
        (append_arg(args), ...);
        return *this;
    }
    void exec() {
        if (bytecodes_.empty()) return;
        asm volatile("" ::: "memory");
        interpreter::stream_exec(bytecodes_.data(), bytecodes_.size());
    }
    void clear() {
        bytecodes_.clear();
        loop_marks_.clear();
    }
    size_t size() const { return bytecodes_.size(); }
    const uint8_t* data() const { return bytecodes_.data(); }
};

}  // namespace ane
