// Warp-level encoders shared by the encode kernels and the fused decode step.
//
// One warp encodes one vector.  Lane l holds elements l + 32k (k < head_dim/32),
// so __ballot_sync(x >= 0) yields sign word k directly (bit i%32 of word i/32,
// reference binary_encode.cu:36-39), and the mean-|x| reduction is evaluated in
// exactly the reference's order: per-thread strided sums over a 128-thread
// block followed by the stride-halving tree (binary_encode.cu:32-50).  Both
// divisions (sum / head_dim and 7 / absmax) are written as in the reference
// with runtime operands and the library is compiled with --use_fast_math like
// the reference, so they lower to the same instruction and the encodings are
// bit-identical.
#pragma once

#include "common.cuh"

namespace bc {

template <int NW>
__device__ __forceinline__ void load_vec(const __half* __restrict__ v, int lane, float (&x)[NW]) {
#pragma unroll
    for (int k = 0; k < NW; ++k) x[k] = __half2float(v[32 * k + lane]);
}

template <int NW>
__device__ __forceinline__ void sign_words(const float (&x)[NW], uint32_t (&w)[NW]) {
#pragma unroll
    for (int k = 0; k < NW; ++k) w[k] = __ballot_sync(0xffffffffu, x[k] >= 0.0f);
}

// Sum of |x_i| in the reference block order (see file comment).  Thread t of
// the reference's 128-thread block owns t and t + 128; here t = lane + 32k.
template <int NW>
__device__ __forceinline__ float tree_abs_sum(const float (&x)[NW]) {
    float p7[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float s = 0.0f;
        if (k < NW) s += fabsf(x[k]);
        if (k + 4 < NW) s += fabsf(x[k + 4]);
        p7[k] = s;
    }
    const float p6a = p7[0] + p7[2];  // stride 64
    const float p6b = p7[1] + p7[3];
    float v = p6a + p6b;              // stride 32
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);  // strides 16..1
    return v;
}

// INT4 residual of x against sign bits w and binary scale s (residual.cu:30-77,
// online_encode.cu:85-119).  Codes are two's complement.
//  PLANE = false (reference records): lanes 4m (m < 8) hold the 16-bit pair of
//    bytes 16k+2m, 16k+2m+1 of the reference byte order in nh[k].
//  PLANE = true (nibble planes), by-bit order (head_dim 64, 128, 256): lanes
//    L < 4 hold in nw[k] the word nib_word(NW, L, k) of nibble_chunk(NW, L, k)
//    (head_dim 128: word k of chunk L; 256: word k % 4 of chunk 4 (k / 4) + L;
//    64: word 2 (L % 2) + k of chunk L / 2); at other head dims lanes 8m
//    (m < 4) hold word m of chunk k in nw[k] (8 codes, element 8j low nibble first).
template <int NW, bool PLANE>
__device__ __forceinline__ float quantise_residual(const float (&x)[NW], const uint32_t (&w)[NW], float s, int lane,
                                                   uint32_t (&nw)[NW], uint32_t (&nh)[NW]) {
    float r[NW];
    float lm = 0.0f;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        const uint32_t bit = (w[k] >> lane) & 1u;
        const float rec = bit ? s : -s;
        r[k] = x[k] - rec;
        lm = fmaxf(lm, fabsf(r[k]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, off));
    const float absmax = lm;
    const float inv_absmax = (absmax > 0.0f) ? (7.0f / absmax) : 0.0f;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        int q = __float2int_rn(r[k] * inv_absmax);
        q = max(-7, min(7, q));
        const uint32_t nb = (uint32_t)q & 0xFu;
        if constexpr (PLANE && nib_by_bit(32 * NW)) {
            // lane l = 8b + L + 4h holds dim 32k + l, i.e. bit L + 4h of sign
            // byte 4k + b; the nibble byte of (sign byte 4k + b, bits L, L + 4)
            // is (lane 8b + L, lane 8b + L + 4), and lane L gathers b = 0..3
            const uint32_t byte = nb | (__shfl_down_sync(0xffffffffu, nb, 4) << 4);
            const uint32_t t1 = byte | (__shfl_down_sync(0xffffffffu, byte, 8) << 8);
            nw[k] = t1 | (__shfl_down_sync(0xffffffffu, t1, 16) << 16);
            nh[k] = 0;
        } else {
            const uint32_t hi = __shfl_down_sync(0xffffffffu, nb, 1);
            const uint32_t byte = nb | (hi << 4);
            const uint32_t t1 = byte | (__shfl_down_sync(0xffffffffu, byte, 2) << 8);
            const uint32_t t2 = t1 | (__shfl_down_sync(0xffffffffu, t1, 4) << 16);
            nh[k] = t1;
            nw[k] = t2;
        }
    }
    return absmax;
}

__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half(f)); }

// ---------------------------------------------------------------------------
// Plane writers
// ---------------------------------------------------------------------------
template <int NW>
__device__ __forceinline__ void store_sign_row(uint32_t* row, const uint32_t (&w)[NW], int lane) {
#pragma unroll
    for (int k = 0; k < NW; ++k)
        if (lane == k) row[k] = w[k];
}

// The nibble chunks of plane row `row` from quantise_residual<NW, true>'s
// words, interleaved layout, stored offset-binary (each nibble holds code + 8).
// By-bit order: where lane L's words go (nibble chunk, first byte of the run),
// the words being consecutive: head_dim 128: nw[0..3] -> chunk L; 256: nw[0..3]
// -> chunk L, nw[4..7] -> chunk 4 + L; 64: nw[0..1] -> chunk L / 2 at byte 8 (L % 2).
template <int NW>
__device__ __forceinline__ void nib_words_to(uint8_t* dst_chunk0, int chunk_stride, const uint32_t (&nw)[NW], int L) {
    if constexpr (NW == 4) {
        *reinterpret_cast<uint4*>(dst_chunk0 + L * chunk_stride) =
            make_uint4(nw[0] ^ 0x88888888u, nw[1] ^ 0x88888888u, nw[2] ^ 0x88888888u, nw[3] ^ 0x88888888u);
    } else if constexpr (NW == 8) {
        *reinterpret_cast<uint4*>(dst_chunk0 + L * chunk_stride) =
            make_uint4(nw[0] ^ 0x88888888u, nw[1] ^ 0x88888888u, nw[2] ^ 0x88888888u, nw[3] ^ 0x88888888u);
        *reinterpret_cast<uint4*>(dst_chunk0 + (4 + L) * chunk_stride) =
            make_uint4(nw[4] ^ 0x88888888u, nw[5] ^ 0x88888888u, nw[6] ^ 0x88888888u, nw[7] ^ 0x88888888u);
    } else {
        static_assert(NW == 2, "by-bit nibble order: head_dim 64, 128 or 256");
        *reinterpret_cast<uint2*>(dst_chunk0 + (L >> 1) * chunk_stride + 8 * (L & 1)) =
            make_uint2(nw[0] ^ 0x88888888u, nw[1] ^ 0x88888888u);
    }
}

template <int NW>
__device__ __forceinline__ void store_nib_row(uint8_t* plane, int64_t row, const uint32_t (&nw)[NW], int lane) {
    if constexpr (nib_by_bit(32 * NW)) {
        if (lane < 4) nib_words_to<NW>(plane + nib_chunk_offset(row, 0, 32 * NW), 128, nw, lane);
    } else {
#pragma unroll
        for (int k = 0; k < NW; ++k)
            if ((lane & 7) == 0)
                *reinterpret_cast<uint32_t*>(plane + nib_chunk_offset(row, k, 32 * NW) + 4 * (lane >> 3)) =
                    nw[k] ^ 0x88888888u;  // offset-binary: code + 8
    }
}

// Encode one vector and hand its pieces to `sink`:
//   sink.sign(w, lane)       every lane holds all NW sign words
//   sink.bscale(bits)        called on lane 0
//   sink.nib(nw, lane)       nibble words as quantise_residual<NW, true> leaves them (two's-complement codes)
//   sink.rscale(bits)        called on lane 0
// The plane writer below and the fused decode step (which also stages the
// row in shared memory) are both sinks, so the arithmetic exists once.
template <int NW, int RES, typename Sink>
__device__ __forceinline__ void encode_row(const float (&x)[NW], int lane, int head_dim, Sink& sink) {
    uint32_t w[NW];
    sign_words<NW>(x, w);
    const float mean_abs = tree_abs_sum<NW>(x) / (float)head_dim;
    const uint16_t sb = f2h_bits(mean_abs);
    sink.sign(w, lane);
    if (lane == 0) sink.bscale(sb);
    if (RES != BC_RES_NONE) {
        const float s = (RES == BC_RES_FP16_SCALE) ? __half2float(__ushort_as_half(sb)) : mean_abs;
        uint32_t nw[NW], nh[NW];
        const float absmax = quantise_residual<NW, true>(x, w, s, lane, nw, nh);
        sink.nib(nw, lane);
        if (lane == 0) sink.rscale(f2h_bits(absmax));
    }
}

// Sink writing plane row `row`.
template <int NW>
struct PlaneRowSink {
    bc_kv_planes P;
    int64_t row;
    __device__ __forceinline__ void sign(const uint32_t (&w)[NW], int lane) {
        store_sign_row<NW>(reinterpret_cast<uint32_t*>(P.sign) + row * NW, w, lane);
    }
    __device__ __forceinline__ void bscale(uint16_t b) { reinterpret_cast<uint16_t*>(P.bscale)[row] = b; }
    __device__ __forceinline__ void nib(const uint32_t (&nw)[NW], int lane) {
        store_nib_row<NW>(reinterpret_cast<uint8_t*>(P.nib), row, nw, lane);
    }
    __device__ __forceinline__ void rscale(uint16_t b) { reinterpret_cast<uint16_t*>(P.rscale)[row] = b; }
};

// Encode one vector into plane row `row`.
template <int NW, int RES>
__device__ __forceinline__ void encode_row_planes(const float (&x)[NW], int lane, int head_dim, bc_kv_planes P,
                                                  int64_t row) {
    PlaneRowSink<NW> sink{P, row};
    encode_row<NW, RES>(x, lane, head_dim, sink);
}

// Prefill encode: each warp takes kVecsPerWarp consecutive vectors per step
// and issues all their loads before encoding any of them, so several hundred
// bytes per warp are in flight and the kernel streams at HBM rate instead of
// waiting out one vector's load latency at a time.
constexpr int kVecsPerWarp = 4;

}  // namespace bc
