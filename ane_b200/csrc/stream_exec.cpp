// stream_exec.cpp -- host decoder of the reference bytecode stream.
//
// Replaces the AArch64 dispatch loop of the reference interpreter
// (src/bytecode_interpreter.s:12-40 fetch / jump table, :174-185 exit).  The
// encoding is the one ane::dispatch produces (include/ane/ane.hpp:206-220): one
// opcode byte, then every argument memcpy'd back to back by sizeof, no padding,
// little-endian.  Hot-path opcodes run on the GPU through the synchronous C
// entry points; any other opcode stops the stream with
// ANE_ERR_UNSUPPORTED_OPCODE (the reference has no bounds check at all).
#include <string.h>

#include <string>

#include "../../include/ane_b200.h"

namespace ane_b200 {
void set_status(int code, const std::string& msg);
int ok();
}  // namespace ane_b200

namespace {

struct Reader {
    const uint8_t* p;
    size_t left;
    template <class T>
    T get() {
        T v;
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        left -= sizeof(T);
        return v;
    }
    template <class T>
    T* ptr() {
        return reinterpret_cast<T*>(static_cast<uintptr_t>(get<uint64_t>()));
    }
};

// Payload sizes (bytes after the opcode) of the executed opcodes.
int payload_size(uint8_t op) {
    switch (op) {
        case 0x0D: return 4 + 4 + 24;       // elementwise_scaled_add_fp32: count scale a b out
        case 0x0F: return 4 + 24;           // relu_backward_fp32: count act grad out
        case 0x11: return 8 + 16;           // transpose_fp32: M N src dst
        case 0x12: return 8 + 40;           // softmax_argmax_fp32: batch cols logits probs labels g_out argmax
        case 0x15: return 12 + 4 + 1 + 32;  // dense_fp32: M N K scale flags A B bias C
        case 0x16: return 4 + 24;           // count_matches: count pred labels out
        case 0x18: return 12 + 8 + 1 + 32;  // dense_i8: M N K sa sb flags A Bp bias C
        case 0x19: return 4 + 24;           // quantize_fp32_i8: count src dst scale_out
        case 0x1A: return 4 + 4 + 16;       // dequantize_i8_fp32: count scale src dst
        case 0x1B: return 8 + 16;           // pack_b_i8: K N src dst
        case 0x1C: return 8 + 24;           // quantize_fp32_i8_channelwise: rows cols src dst scales
        case 0x1E: return 12 + 8 + 1 + 32;  // dense_u8s8: as dense_i8, A unsigned
        case 0x61:                          // cblas_igemm / ugemm / usgemm:
        case 0x62:                          //   flags M N K lda ldb ldc alpha beta A B C
        case 0x63: return 1 + 12 + 12 + 8 + 24;
        case 0x57: return 8 + 24;           // q8_0_gemv: M K in W out
        case 0x58: return 8 + 24;           // q4_0_gemv: M K in W out
        case 0x75:                          // q4_k_gemv: M K in W out
        case 0x76:                          // q2_k_gemv
        case 0x77:                          // q3_k_gemv
        case 0x78:                          // q5_k_gemv
        case 0x79: return 8 + 24;           // q6_k_gemv
        case 0x7C: return 8 + 24;           // get_rows_q8_0: n_rows dim table indices out
        case 0x7D: return 8 + 24;           // get_rows_q4_0: n_rows dim table indices out
        case 0x80: return 12 + 4 + 1 + 24;  // dense_fused_i8: M N K scale relu A B C
        default: return -1;
    }
}

inline uint32_t round16(uint32_t v) { return (v + 15u) & ~15u; }

int exec_one(uint8_t op, Reader& r) {
    switch (op) {
        case 0x0D: {
            uint32_t count = r.get<uint32_t>();
            float scale = r.get<float>();
            const float* a = r.ptr<const float>();
            const float* b = r.ptr<const float>();
            float* out = r.ptr<float>();
            return ane_elementwise_scaled_add_fp32(count, scale, a, b, out);
        }
        case 0x0F: {
            uint32_t count = r.get<uint32_t>();
            const float* act = r.ptr<const float>();
            const float* grad = r.ptr<const float>();
            float* out = r.ptr<float>();
            return ane_relu_backward_fp32(count, act, grad, out);
        }
        case 0x11: {
            uint32_t M = r.get<uint32_t>(), N = r.get<uint32_t>();
            const float* src = r.ptr<const float>();
            float* dst = r.ptr<float>();
            return ane_transpose_fp32(M, N, src, dst);
        }
        case 0x12: {
            uint32_t batch = r.get<uint32_t>(), cols = r.get<uint32_t>();
            const float* logits = r.ptr<const float>();
            float* probs = r.ptr<float>();
            const uint8_t* labels = r.ptr<const uint8_t>();
            float* g_out = r.ptr<float>();
            int32_t* argmax = r.ptr<int32_t>();
            return ane_softmax_argmax_fp32(batch, cols, logits, probs, labels, g_out, argmax);
        }
        case 0x15: {
            uint32_t M = r.get<uint32_t>(), N = r.get<uint32_t>(), K = r.get<uint32_t>();
            float scale = r.get<float>();
            uint8_t flags = r.get<uint8_t>();
            const float* A = r.ptr<const float>();
            const float* B = r.ptr<const float>();
            const float* bias = r.ptr<const float>();
            float* C = r.ptr<float>();
            return ane_dense_fp32(M, N, K, scale, flags, A, B, bias, C);
        }
        case 0x16: {
            uint32_t count = r.get<uint32_t>();
            const int32_t* pred = r.ptr<const int32_t>();
            const uint8_t* labels = r.ptr<const uint8_t>();
            int32_t* out = r.ptr<int32_t>();
            return ane_count_matches(count, pred, labels, out);
        }
        case 0x18: {
            uint32_t M = r.get<uint32_t>(), N = r.get<uint32_t>(), K = r.get<uint32_t>();
            float sa = r.get<float>(), sb = r.get<float>();
            uint8_t flags = r.get<uint8_t>();
            const int8_t* A = r.ptr<const int8_t>();
            const int8_t* Bp = r.ptr<const int8_t>();
            const float* bias = r.ptr<const float>();
            float* C = r.ptr<float>();
            return ane_dense_i8(M, N, K, sa, sb, flags, A, Bp, bias, C);
        }
        case 0x1E: {
            uint32_t M = r.get<uint32_t>(), N = r.get<uint32_t>(), K = r.get<uint32_t>();
            float sa = r.get<float>(), sb = r.get<float>();
            uint8_t flags = r.get<uint8_t>();
            const uint8_t* A = r.ptr<const uint8_t>();
            const int8_t* Bp = r.ptr<const int8_t>();
            const float* bias = r.ptr<const float>();
            float* C = r.ptr<float>();
            return ane_dense_u8s8(M, N, K, sa, sb, flags, A, Bp, bias, C);
        }
        case 0x58: {
            uint32_t M = r.get<uint32_t>(), K = r.get<uint32_t>();
            const float* in = r.ptr<const float>();
            const void* W = r.ptr<const void>();
            float* out = r.ptr<float>();
            return ane_q4_0_gemv(M, K, in, W, out);
        }
        case 0x75:
        case 0x76:
        case 0x77:
        case 0x78:
        case 0x79: {
            uint32_t M = r.get<uint32_t>(), K = r.get<uint32_t>();
            const float* in = r.ptr<const float>();
            const void* W = r.ptr<const void>();
            float* out = r.ptr<float>();
            switch (op) {
                case 0x75: return ane_q4_k_gemv(M, K, in, W, out);
                case 0x76: return ane_q2_k_gemv(M, K, in, W, out);
                case 0x77: return ane_q3_k_gemv(M, K, in, W, out);
                case 0x78: return ane_q5_k_gemv(M, K, in, W, out);
                default: return ane_q6_k_gemv(M, K, in, W, out);
            }
        }
        case 0x7D: {
            uint32_t n_rows = r.get<uint32_t>(), dim = r.get<uint32_t>();
            const void* table = r.ptr<const void>();
            const uint32_t* indices = r.ptr<const uint32_t>();
            float* out = r.ptr<float>();
            return ane_get_rows_q4_0(n_rows, dim, table, indices, out);
        }
        case 0x7C: {
            uint32_t n_rows = r.get<uint32_t>(), dim = r.get<uint32_t>();
            const void* table = r.ptr<const void>();
            const uint32_t* indices = r.ptr<const uint32_t>();
            float* out = r.ptr<float>();
            return ane_get_rows_q8_0(n_rows, dim, table, indices, out);
        }
        case 0x61:
        case 0x62:
        case 0x63: {
            uint8_t flags = r.get<uint8_t>();
            uint32_t M = r.get<uint32_t>(), N = r.get<uint32_t>(), K = r.get<uint32_t>();
            uint32_t lda = r.get<uint32_t>(), ldb = r.get<uint32_t>(), ldc = r.get<uint32_t>();
            float alpha = r.get<float>(), beta = r.get<float>();
            const void* A = r.ptr<const void>();
            const void* B = r.ptr<const void>();
            float* C = r.ptr<float>();
            if (op == 0x61) return ane_cblas_igemm(flags, M, N, K, lda, ldb, ldc, alpha, beta, A, B, C);
            if (op == 0x62) return ane_cblas_ugemm(flags, M, N, K, lda, ldb, ldc, alpha, beta, A, B, C);
            return ane_cblas_usgemm(flags, M, N, K, lda, ldb, ldc, alpha, beta, A, B, C);
        }
        case 0x19: {
            // The handler works on whole 16-lane vectors: ceil(count/16)*16 elements
            // (callers pad buffers to 16 elements, README.md:79).
            uint32_t count = r.get<uint32_t>();
            const float* src = r.ptr<const float>();
            int8_t* dst = r.ptr<int8_t>();
            float* scale_out = r.ptr<float>();
            return ane_quantize_fp32_i8(round16(count), src, dst, scale_out);
        }
        case 0x1A: {
            uint32_t count = r.get<uint32_t>();
            float scale = r.get<float>();
            const int8_t* src = r.ptr<const int8_t>();
            float* dst = r.ptr<float>();
            return ane_dequantize_i8_fp32(count, scale, src, dst);
        }
        case 0x1B: {
            uint32_t K = r.get<uint32_t>(), N = r.get<uint32_t>();
            const int8_t* src = r.ptr<const int8_t>();
            int8_t* dst = r.ptr<int8_t>();
            return ane_pack_b_i8(K, N, src, dst);
        }
        case 0x1C: {
            // rows are walked contiguously in whole 16-element vectors
            uint32_t rows = r.get<uint32_t>(), cols = r.get<uint32_t>();
            const float* src = r.ptr<const float>();
            int8_t* dst = r.ptr<int8_t>();
            float* scales = r.ptr<float>();
            return ane_quantize_fp32_i8_channelwise(rows, round16(cols), src, dst, scales);
        }
        case 0x57: {
            uint32_t M = r.get<uint32_t>(), K = r.get<uint32_t>();
            const float* in = r.ptr<const float>();
            const void* W = r.ptr<const void>();
            float* out = r.ptr<float>();
            return ane_q8_0_gemv(M, K & ~31u, in, W, out);  // num_blocks = K/32
        }
        case 0x80: {
            uint32_t M = r.get<uint32_t>(), N = r.get<uint32_t>(), K = r.get<uint32_t>();
            float scale = r.get<float>();
            uint8_t relu = r.get<uint8_t>();
            const float* A = r.ptr<const float>();
            const float* B = r.ptr<const float>();
            float* C = r.ptr<float>();
            return ane_dense_fused_i8(M, N, K, scale, relu ? 1 : 0, A, B, C);
        }
        default:
            return ANE_ERR_UNSUPPORTED_OPCODE;
    }
}

}  // namespace

extern "C" {

int ane_opcode_payload_size(uint8_t op) { return payload_size(op); }
int ane_opcode_supported(uint8_t op) { return payload_size(op) >= 0 ? 1 : 0; }

void stream_exec(const uint8_t* data, size_t size) {
    using namespace ane_b200;
    if (size && !data) {
        set_status(ANE_ERR_INVALID_ARGUMENT, "stream_exec: NULL stream");
        return;
    }
    Reader r{data, size};
    while (r.left > 0) {
        const uint8_t op = r.get<uint8_t>();
        if (op == 0x00) break;  // reserved slot 0 = exit (jump table entry 0)
        const int need = payload_size(op);
        if (need < 0) {
            set_status(ANE_ERR_UNSUPPORTED_OPCODE,
                       "stream_exec: opcode 0x" + std::to_string(op) + " is outside the B200 hot path");
            return;
        }
        if ((size_t)need > r.left) {
            set_status(ANE_ERR_TRUNCATED_STREAM, "stream_exec: payload of opcode " + std::to_string(op) +
                                                     " runs past the end of the stream");
            return;
        }
        const int rc = exec_one(op, r);
        if (rc != ANE_OK) return;  // the entry point recorded the detail
    }
    ok();
}

}  // extern "C"
