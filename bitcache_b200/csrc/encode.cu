// Encoders: sign-bit packing + mean|x| scale, INT4 residual, online (decode
// step) append, and record <-> plane converters.  sm_100a.
//
// The warp-level encoders themselves live in encode_core.cuh (one warp per
// vector, reference summation order, bit-identical to the reference kernels).
#include "encode_core.cuh"

namespace bc {

// ---------------------------------------------------------------------------
// Reference-record writers
// ---------------------------------------------------------------------------
template <int NW>
__device__ __forceinline__ void store_binvec(uint8_t* rec, const uint32_t (&w)[NW], uint16_t scale, int lane) {
    uint32_t* rw = reinterpret_cast<uint32_t*>(rec);
    if (lane < 8) {
        uint32_t v = 0;
#pragma unroll
        for (int k = 0; k < NW; ++k)
            if (lane == k) v = w[k];
        rw[lane] = v;  // words NW..7 zeroed
    } else if (lane == 8) {
        rw[8] = (uint32_t)scale;  // scale + zeroed padding
    }
}

template <int NW>
__device__ __forceinline__ void store_resvec(uint8_t* rec, const uint32_t (&nh)[NW], uint16_t scale, int lane) {
    uint16_t* rh = reinterpret_cast<uint16_t*>(rec);  // records are 2-byte aligned
#pragma unroll
    for (int k = 0; k < NW; ++k)
        if ((lane & 3) == 0) rh[8 * k + (lane >> 2)] = (uint16_t)nh[k];
    for (int i = 8 * NW + lane; i < 64; i += 32) rh[i] = 0;  // unused nibbles zeroed
    if (lane == 0) rh[64] = scale;
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
constexpr int kEncWarps = 8;

template <int NW>
__global__ void __launch_bounds__(kEncWarps * 32) k_binary_encode_rec(const __half* __restrict__ src,
                                                                      uint8_t* __restrict__ out, int64_t n,
                                                                      int head_dim) {
    const int lane = threadIdx.x & 31;
    const int64_t v = (int64_t)blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (v >= n) return;
    float x[NW];
    load_vec<NW>(src + v * head_dim, lane, x);
    uint32_t w[NW];
    sign_words<NW>(x, w);
    const float mean_abs = tree_abs_sum<NW>(x) / (float)head_dim;
    store_binvec<NW>(out + v * kBinRecBytes, w, f2h_bits(mean_abs), lane);
}

template <int NW>
__global__ void __launch_bounds__(kEncWarps * 32) k_residual_encode_rec(const __half* __restrict__ src,
                                                                        const uint8_t* __restrict__ bin,
                                                                        uint8_t* __restrict__ out, int64_t n,
                                                                        int head_dim) {
    const int lane = threadIdx.x & 31;
    const int64_t v = (int64_t)blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (v >= n) return;
    float x[NW];
    load_vec<NW>(src + v * head_dim, lane, x);
    const uint8_t* brec = bin + v * kBinRecBytes;
    uint32_t w[NW];
#pragma unroll
    for (int k = 0; k < NW; ++k) w[k] = reinterpret_cast<const uint32_t*>(brec)[k];
    const float s = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(brec + kBinScaleOff)));
    uint32_t nw[NW], nh[NW];
    const float absmax = quantise_residual<NW, false>(x, w, s, lane, nw, nh);
    store_resvec<NW>(out + v * kResRecBytes, nh, f2h_bits(absmax), lane);
}

// Online token encode into reference-record ring buffers (online_encode.cu:17-120).
template <int NW>
__global__ void __launch_bounds__(kEncWarps * 32) k_online_encode_rec(const __half* __restrict__ kv,
                                                                      uint8_t* __restrict__ bin,
                                                                      uint8_t* __restrict__ res, int n_slots,
                                                                      int head_dim, int write_slot, int max_seq) {
    const int lane = threadIdx.x & 31;
    const int slot = blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (slot >= n_slots) return;
    float x[NW];
    load_vec<NW>(kv + (int64_t)slot * head_dim, lane, x);
    uint32_t w[NW];
    sign_words<NW>(x, w);
    const float scale_bin = tree_abs_sum<NW>(x) / (float)head_dim;
    const int64_t cache_idx = (int64_t)slot * max_seq + write_slot;
    store_binvec<NW>(bin + cache_idx * kBinRecBytes, w, f2h_bits(scale_bin), lane);
    if (res != nullptr) {
        uint32_t nw[NW], nh[NW];
        const float absmax = quantise_residual<NW, false>(x, w, scale_bin, lane, nw, nh);
        store_resvec<NW>(res + cache_idx * kResRecBytes, nh, f2h_bits(absmax), lane);
    }
}

template <int NW, int RES>
__global__ void __launch_bounds__(kEncWarps * 32) k_encode_planes(const __half* __restrict__ src, bc_kv_planes P,
                                                                  int n_slots, int seq_len, int64_t kv_stride,
                                                                  int head_dim) {
    const int lane = threadIdx.x & 31;
    const int64_t n = (int64_t)n_slots * seq_len;
    const int64_t nwarps = (int64_t)gridDim.x * kEncWarps;
    for (int64_t v0 = ((int64_t)blockIdx.x * kEncWarps + (threadIdx.x >> 5)) * kVecsPerWarp; v0 < n;
         v0 += nwarps * kVecsPerWarp) {
        float x[kVecsPerWarp][NW];
#pragma unroll
        for (int j = 0; j < kVecsPerWarp; ++j)
            if (v0 + j < n) load_vec<NW>(src + (v0 + j) * head_dim, lane, x[j]);
#pragma unroll
        for (int j = 0; j < kVecsPerWarp; ++j) {
            const int64_t v = v0 + j;
            if (v >= n) break;  // warp-uniform
            const int64_t slot = v / seq_len, s = v - slot * seq_len;
            encode_row_planes<NW, RES>(x[j], lane, head_dim, P, slot * kv_stride + s);
        }
    }
}

// ---------------------------------------------------------------------------
// Prefill encode, one vector per lane (head_dim <= 128).  The per-warp encoder
// above spends ~6 shuffles and ballots per 32 elements; here each lane owns a
// whole vector, so the arithmetic is the same per element but nothing crosses
// lanes.  Every lane copies its fp16 row (one 1-D bulk copy) into a padded
// shared-memory row of its warp's double buffer, so the 16-byte reads that
// follow spread over all banks.  The mean-|x| sum is evaluated in the
// reference's block-tree order (leaf t = |x_t|, strides 64, 32, ..., 1), depth
// first so that only one partial per level is live; the residual uses the
// same operations as quantise_residual (fast-math 7/absmax, cvt.rni, clamp),
// so the planes are bit-identical to the per-warp encoder's.
// ---------------------------------------------------------------------------
constexpr int kLpvWarps = 4;

template <int D>
struct LpvCfg {
    static constexpr int ROWB = 2 * D + 16;         // padded row: consecutive lanes start 16 B apart in bank terms
    static constexpr int BUFB = 32 * ROWB;          // one batch of 32 vectors
    static constexpr int WARPB = 2 * BUFB + 16;     // double buffer + 2 mbarriers
    static constexpr int SMEM_B = kLpvWarps * WARPB + 128;
};

// Eight fp32 values of one 16-byte chunk of fp16 elements.
__device__ __forceinline__ void lpv_chunk(const uint4& t, float (&x)[8]) {
    const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

// The reference's 128-leaf stride-halving tree (leaf t = |x_t|, 0 beyond
// head_dim; strides 64, 32, ..., 1), split by the position j = t % 8 within a
// 16-byte chunk k = t / 8: strides 64, 32, 16, 8 pair chunks differing in bit
// 3, 2, 1, 0 of k, so for each j the partial after stride 8 is the same tree
// over the 16 chunks, whose root joins the chunks differing in bit 0.
// lpv_tree16 walks it depth first (level L joins chunks differing in bit L;
// one chunk read per leaf, four levels live); strides 4, 2, 1 then combine
// the eight per-position partials.
template <int D, int L, int K>
__device__ __forceinline__ void lpv_tree16(const uint4* row, float (&out)[8]) {
    if constexpr (L == 4) {  // leaf: chunk K
        if constexpr (8 * K >= D) {
#pragma unroll
            for (int j = 0; j < 8; ++j) out[j] = 0.0f;
        } else {
            float x[8];
            lpv_chunk(row[K], x);
#pragma unroll
            for (int j = 0; j < 8; ++j) out[j] = fabsf(x[j]);
        }
    } else if constexpr (8 * (K + (1 << L)) >= D) {
        // the right subtree covers chunks beyond head_dim only: adding +0.0f is exact for a >= 0
        lpv_tree16<D, L + 1, K>(row, out);
    } else {
        float right[8];
        lpv_tree16<D, L + 1, K>(row, out);
        lpv_tree16<D, L + 1, K + (1 << L)>(row, right);
#pragma unroll
        for (int j = 0; j < 8; ++j) out[j] += right[j];
    }
}

template <int D>
__device__ __forceinline__ float lpv_abs_sum(const uint4* row) {
    float a[8];
    lpv_tree16<D, 0, 0>(row, a);
    const float u0 = a[0] + a[4], u1 = a[1] + a[5], u2 = a[2] + a[6], u3 = a[3] + a[7];  // stride 4
    const float v0 = u0 + u2, v1 = u1 + u3;                                              // stride 2
    return v0 + v1;                                                                      // stride 1
}

// ---- head_dim 64 and 128 (by-bit nibble order): two passes over the row ----
// Pass 1 sums |x| in the reference's tree order (as lpv_tree16) and also keeps
// min |x| and max |x| (fp16, exact).  The residual's absmax needs no pass of
// its own: |x - rec| = |fl(|x| - sc)| for every element (rec = +sc for
// x >= 0, -sc otherwise, and RN is symmetric), and fl(a - sc) is monotone in
// a, so the largest |x - rec| is reached at min |x| or at max |x|.  With a NaN
// element sc is NaN and both terms are NaN, which fmaxf drops, as the
// reference's per-element fmaxf does.  Pass 2 builds the sign bits and the
// INT4 codes with packed fp32x2 arithmetic, in the by-bit nibble order.
__device__ __forceinline__ float2 add2_ftz(float2 a, float2 b) {
    unsigned long long r;
    asm("add.rn.ftz.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)));
    return *reinterpret_cast<float2*>(&r);
}
__device__ __forceinline__ float2 mul2_ftz(float2 a, float2 b) {
    unsigned long long r;
    asm("mul.rn.ftz.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)));
    return *reinterpret_cast<float2*>(&r);
}
// 0xFFFF in each half where that fp16 element is >= 0 (so -0 is, NaN is not).
__device__ __forceinline__ uint32_t hge0_mask(uint32_t h2) {
    uint32_t m;
    asm("set.ge.u32.f16x2 %0, %1, %2;" : "=r"(m) : "r"(h2), "r"(0u));
    return m;
}
__device__ __forceinline__ uint32_t bfi32(uint32_t src, uint32_t base, uint32_t pos, uint32_t len) {
    uint32_t r;
    asm("bfi.b32 %0, %1, %2, %3, %4;" : "=r"(r) : "r"(src), "r"(base), "r"(pos), "r"(len));
    return r;
}
// Four per-element flags (0xFFFF / 0 halves of a, then b) as bits 0..3: the
// high bytes of the halves gathered by one byte permute, their top bits moved
// to bits 28..31 by one multiply (the four partial products land on distinct
// bits, so no carries).
__device__ __forceinline__ uint32_t flags4(uint32_t a, uint32_t b) {
    return ((__byte_perm(a, b, 0x7531) & 0x80808080u) * 0x00204081u) >> 28;
}
__device__ __forceinline__ uint4 lds128_volatile(const void* p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(smem_u32(p)) : "memory");
    return r;
}
__device__ __forceinline__ void sts32_volatile(void* p, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ float2 h2_to_f2(uint32_t h2) {
    return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}

template <int D, int L, int K>
__device__ __forceinline__ void lpv_tree16_mm(const uint4* row, float (&out)[8], __half2& mx, __half2& mn) {
    if constexpr (L == 4 && 8 * K >= D) {  // leaf beyond head_dim: zeros
#pragma unroll
        for (int j = 0; j < 8; ++j) out[j] = 0.0f;
    } else if constexpr (L == 4) {  // leaf: chunk K
        const uint4 t = row[K];
        const uint32_t w[4] = {t.x & 0x7FFF7FFFu, t.y & 0x7FFF7FFFu, t.z & 0x7FFF7FFFu, t.w & 0x7FFF7FFFu};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            mx = __hmax2(mx, h);
            mn = __hmin2(mn, h);
            const float2 f = __half22float2(h);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    } else if constexpr (8 * (K + (1 << L)) >= D) {
        // the right subtree covers chunks beyond head_dim only: adding +0.0f is exact for a >= 0
        lpv_tree16_mm<D, L + 1, K>(row, out, mx, mn);
    } else {
        float right[8];
        lpv_tree16_mm<D, L + 1, K>(row, out, mx, mn);
        lpv_tree16_mm<D, L + 1, K + (1 << L)>(row, right, mx, mn);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 s = add2_ftz(make_float2(out[2 * i], out[2 * i + 1]), make_float2(right[2 * i], right[2 * i + 1]));
            out[2 * i] = s.x;
            out[2 * i + 1] = s.y;
        }
    }
}

template <int D, int RES>
__device__ __forceinline__ void lpv_encode_row_bybit(const uint4* row, bc_kv_planes P, int64_t v, int seq_len,
                                                     int64_t kv_stride, int head_dim) {
    static_assert(D == 64 || D == 128, "one vector per lane: head_dim 64 or 128");
    constexpr int NW = D / 32;
    float a[8];
    __half2 mx = __float2half2_rn(0.0f), mn = __float2half2_rn(INFINITY);
    lpv_tree16_mm<D, 0, 0>(row, a, mx, mn);
    const float u0 = a[0] + a[4], u1 = a[1] + a[5], u2 = a[2] + a[6], u3 = a[3] + a[7];  // stride 4
    const float v0 = u0 + u2, v1 = u1 + u3;                                              // stride 2
    const float mean_abs = (v0 + v1) / (float)head_dim;                                  // stride 1
    const uint16_t sb = f2h_bits(mean_abs);
    const float sc = (RES == BC_RES_FP16_SCALE) ? __half2float(__ushort_as_half(sb)) : mean_abs;
    float absmax = 0.0f;
    if constexpr (RES != BC_RES_NONE) {
        const float lo = fminf(__low2float(mn), __high2float(mn)), hi = fmaxf(__low2float(mx), __high2float(mx));
        absmax = fmaxf(fmaxf(0.0f, fabsf(lo - sc)), fabsf(hi - sc));
    }
    const float inv_absmax = (absmax > 0.0f) ? (7.0f / absmax) : 0.0f;
    // See lpv_encode_row_small for the rounding by adding 1.5 * 2^23.
    constexpr float kRound = 12582912.0f;
    const float2 nsc = make_float2(-sc, -sc), inv2 = make_float2(inv_absmax, inv_absmax),
                 rnd2 = make_float2(kRound, kRound);
    const bool live = inv_absmax > 0.0f;
    // Four input chunks (sign byte j = 4w .. 4w + 3: dims 8j .. 8j + 7) per
    // step.  Element r of input chunk j is bit r of sign byte j; its code goes
    // to nibble r / 4 of the nibble byte of (j, t = r % 4), which this step
    // collects in cur[t]: head_dim 128: word w of chunk t; head_dim 64: word
    // 2 (t % 2) + w of chunk t / 2.  The loads and the stores of finished
    // words are volatile, so the compiler keeps one step's 16 input words
    // live, not the whole row's.  Finished words go back into the row's first
    // D / 2 bytes (input chunks no longer read), in chunk order.
    uint8_t* rb = reinterpret_cast<uint8_t*>(const_cast<uint4*>(row));
    uint32_t sw[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        uint32_t cur[4] = {0u, 0u, 0u, 0u};
        uint32_t sword = 0u;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {  // input chunk j = 4w + jj: dims 8j .. 8j + 7
            const int j = 4 * w + jj;
            const uint4 t = lds128_volatile(rb + 16 * j);
            const uint32_t h[4] = {t.x, t.y, t.z, t.w};
            uint32_t m[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) m[i] = hge0_mask(h[i]);
            sword = bfi32(flags4(m[0], m[1]) | (flags4(m[2], m[3]) << 4), sword, 8 * jj, 8);
            if constexpr (RES != BC_RES_NONE) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {  // elements 2i, 2i + 1
                    // (|x| - sc) * inv, negated for x < 0: the rounded (x - rec) * inv_absmax
                    float2 p = mul2_ftz(add2_ftz(h2_to_f2(h[i] & 0x7FFF7FFFu), nsc), inv2);
                    p.x = __uint_as_float(__float_as_uint(p.x) ^ ((~m[i] << 16) & 0x80000000u));
                    p.y = __uint_as_float(__float_as_uint(p.y) ^ (~m[i] & 0x80000000u));
                    const float2 q = add2_ftz(p, rnd2);
                    const int e0 = 2 * i, e1 = 2 * i + 1;  // element e: word cur[e % 4], high nibble for e >= 4
                    cur[e0 & 3] = bfi32(__float_as_uint(q.x), cur[e0 & 3], 8 * jj + 4 * (e0 >> 2), 4);
                    cur[e1 & 3] = bfi32(__float_as_uint(q.y), cur[e1 & 3], 8 * jj + 4 * (e1 >> 2), 4);
                }
            }
        }
        sw[w] = sword;
        if constexpr (RES != BC_RES_NONE) {
#pragma unroll
            for (int t = 0; t < 4; ++t)  // byte offset of the word in chunk order: 16t + 4w (128), 8t + 4w (64)
                sts32_volatile(rb + (D == 128 ? 16 : 8) * t + 4 * w, live ? cur[t] ^ 0x88888888u : 0x88888888u);
        }
    }
    const int64_t slot = v / seq_len, pos = v - slot * seq_len;
    const int64_t r = slot * kv_stride + pos;
    if constexpr (NW == 4)
        *reinterpret_cast<uint4*>(reinterpret_cast<uint32_t*>(P.sign) + r * 4) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
    else
        *reinterpret_cast<uint2*>(reinterpret_cast<uint32_t*>(P.sign) + r * 2) = make_uint2(sw[0], sw[1]);
    reinterpret_cast<uint16_t*>(P.bscale)[r] = sb;
    if constexpr (RES != BC_RES_NONE) {
        uint8_t* nb = reinterpret_cast<uint8_t*>(P.nib);
#pragma unroll
        for (int c = 0; c < NW; ++c)
            *reinterpret_cast<uint4*>(nb + nib_chunk_offset(r, c, D)) = lds128_volatile(rb + 16 * c);
        reinterpret_cast<uint16_t*>(P.rscale)[r] = f2h_bits(absmax);
    }
}

// Encode the vector in shared-memory row `row` into plane row v (lane-local),
// head dims 32 and 96 (reference nibble order): three passes over the row.
template <int NW, int RES>
__device__ __forceinline__ void lpv_encode_row_small(const uint4* row, bc_kv_planes P, int64_t v, int seq_len,
                                                     int64_t kv_stride, int head_dim) {
    constexpr int D = 32 * NW;
    static_assert(!nib_by_bit(D), "head dims 64 and 128 have their own row encoder");
    const float mean_abs = lpv_abs_sum<D>(row) / (float)head_dim;
    const uint16_t sb = f2h_bits(mean_abs);
    const float sc = (RES == BC_RES_FP16_SCALE) ? __half2float(__ushort_as_half(sb)) : mean_abs;
    // signs (x >= 0, so -0 -> 1 and NaN -> 0) and the residual absmax in one pass
    uint32_t w[NW];
    float absmax = 0.0f;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float x[8];
            lpv_chunk(row[4 * k + c], x);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool bit = x[j] >= 0.0f;
                word |= (bit ? 1u : 0u) << (8 * c + j);
                if (RES != BC_RES_NONE) absmax = fmaxf(absmax, fabsf(x[j] - (bit ? sc : -sc)));
            }
        }
        w[k] = word;
    }
    const int64_t slot = v / seq_len, pos = v - slot * seq_len;
    const int64_t r = slot * kv_stride + pos;
    uint32_t* srow = reinterpret_cast<uint32_t*>(P.sign) + r * NW;
    if constexpr (NW == 4) {
        *reinterpret_cast<uint4*>(srow) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if constexpr (NW == 2) {
        *reinterpret_cast<uint2*>(srow) = make_uint2(w[0], w[1]);
    } else {
#pragma unroll
        for (int k = 0; k < NW; ++k) srow[k] = w[k];
    }
    reinterpret_cast<uint16_t*>(P.bscale)[r] = sb;
    if constexpr (RES != BC_RES_NONE) {
        const float inv_absmax = (absmax > 0.0f) ? (7.0f / absmax) : 0.0f;
        // Rounding.  With inv_absmax > 0 the scale is finite and every r finite
        // with |r * inv_absmax| <= 7 (to a few ulp), so adding 1.5 * 2^23 rounds
        // to the nearest integer, ties to even, exactly as cvt.rni, and leaves
        // the code's two's complement in the low 4 bits; the reference's clamp
        // to [-7, 7] never binds.  inv_absmax == 0 (zero, NaN or infinite input)
        // gives code 0 everywhere, as cvt.rni of 0 or NaN does.
        const bool live = inv_absmax > 0.0f;
        constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
        uint8_t* nb = reinterpret_cast<uint8_t*>(P.nib);
#pragma unroll
        for (int k = 0; k < NW; ++k) {
            uint32_t wd[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float x[8];
                lpv_chunk(row[4 * k + c], x);
                uint32_t word = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float rec = ((w[k] >> (8 * c + j)) & 1u) ? sc : -sc;
                    // __fmul_rn: the product is rounded to fp32 first, as before cvt.rni
                    // (a contracted fma would round the exact product instead)
                    const uint32_t q = __float_as_uint(__fadd_rn(__fmul_rn(x[j] - rec, inv_absmax), kRound));
                    word |= (q & 0xFu) << (4 * j);
                }
                wd[c] = live ? word ^ 0x88888888u : 0x88888888u;  // offset-binary: code + 8
            }
            *reinterpret_cast<uint4*>(nb + nib_chunk_offset(r, k, D)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
        reinterpret_cast<uint16_t*>(P.rscale)[r] = f2h_bits(absmax);
    }
}

template <int NW, int RES>
__device__ __forceinline__ void lpv_encode_row(const uint4* row, bc_kv_planes P, int64_t v, int seq_len,
                                               int64_t kv_stride, int head_dim) {
    if constexpr (nib_by_bit(32 * NW))
        lpv_encode_row_bybit<32 * NW, RES>(row, P, v, seq_len, kv_stride, head_dim);
    else
        lpv_encode_row_small<NW, RES>(row, P, v, seq_len, kv_stride, head_dim);
}

template <int NW, int RES>
__global__ void __launch_bounds__(kLpvWarps * 32, 3) k_encode_planes_lpv(const __half* __restrict__ src, bc_kv_planes P,
                                                                      int seq_len, int64_t kv_stride, int head_dim,
                                                                      int64_t n, unsigned int* err) {
    constexpr int D = 32 * NW;
    using C = LpvCfg<D>;
    extern __shared__ __align__(128) uint8_t lpv_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(lpv_raw) + 127) & ~uintptr_t(127));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint8_t* wbuf = smem + warp * C::WARPB;
    uint64_t* full = reinterpret_cast<uint64_t*>(wbuf + 2 * C::BUFB);
    const int64_t n_batches = (n + 31) / 32;
    const int64_t stride_b = (int64_t)gridDim.x * kLpvWarps;
    const int64_t first = (int64_t)blockIdx.x * kLpvWarps + warp;
    if (lane == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    __syncwarp();
    auto issue = [&](int64_t b, int buf) {
        const int cnt = (int)min((int64_t)32, n - 32 * b);
        if (lane == 0) mbar_arrive_expect_tx(&full[buf], (uint32_t)cnt * 2 * D);
        __syncwarp();
        if (lane < cnt)
            bulk_g2s(wbuf + buf * C::BUFB + lane * C::ROWB, src + (32 * b + lane) * D, 2 * D, &full[buf]);
    };
    if (first < n_batches) issue(first, 0);
    if (first + stride_b < n_batches) issue(first + stride_b, 1);
    int it = 0;
    for (int64_t b = first; b < n_batches; b += stride_b, ++it) {
        const int buf = it & 1;
        if (!mbar_wait_bounded(&full[buf], (uint32_t)(it >> 1) & 1u)) {
            if (lane == 0) raise_device_error(err, BC_DEVERR_TIMEOUT);
            // drain what is still in flight (bounded), then leave
            if (b + stride_b < n_batches) mbar_wait_bounded(&full[buf ^ 1], (uint32_t)((it + 1) >> 1) & 1u);
            return;
        }
        const int64_t v = 32 * b + lane;
        if (v < n) {
            const uint4* row = reinterpret_cast<const uint4*>(wbuf + buf * C::BUFB + lane * C::ROWB);
            lpv_encode_row<NW, RES>(row, P, v, seq_len, kv_stride, head_dim);
        }
        __syncwarp();
        // the buffer is read: refill it with the batch two steps ahead
        if (b + 2 * stride_b < n_batches) {
            fence_proxy_async_smem();
            issue(b + 2 * stride_b, buf);
        }
    }
}

// Append one K and one V token per slot: warps [0, n_slots) encode K, the rest V.
template <int NW, int RES>
__global__ void __launch_bounds__(kEncWarps * 32) k_append_kv(const __half* __restrict__ k,
                                                              const __half* __restrict__ v, bc_kv_planes K,
                                                              bc_kv_planes V, int n_slots, int head_dim,
                                                              int64_t kv_stride, int64_t pos, bc_page_table pt,
                                                              unsigned int* err) {
    const int lane = threadIdx.x & 31;
    const int wid = blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (wid >= 2 * n_slots) return;
    const bool is_v = wid >= n_slots;
    const int slot = is_v ? wid - n_slots : wid;
    int64_t row = (int64_t)slot * kv_stride + pos;
    if (pt.pages) {  // paged cache: the block table names the page
        const int pg = __ldg(pt.pages + (int64_t)slot * pt.max_pages + pos / pt.page_size);
        if (pg < 0 || pg >= pt.n_pages) {
            if (lane == 0 && err) raise_device_error(err, BC_DEVERR_PAGE);
            return;
        }
        row = (int64_t)pg * pt.page_size + pos % pt.page_size;
    }
    float x[NW];
    load_vec<NW>((is_v ? v : k) + (int64_t)slot * head_dim, lane, x);
    encode_row_planes<NW, RES>(x, lane, head_dim, is_v ? V : K, row);
}

// Record <-> plane conversion (pure data movement, one warp per vector).
template <int NW>
__global__ void __launch_bounds__(kEncWarps * 32) k_records_to_planes(const uint8_t* __restrict__ bin,
                                                                      const uint8_t* __restrict__ res,
                                                                      bc_kv_planes P, int64_t n) {
    const int lane = threadIdx.x & 31;
    const int64_t v = (int64_t)blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (v >= n) return;
    const uint8_t* b = bin + v * kBinRecBytes;
    if (lane < NW) reinterpret_cast<uint32_t*>(P.sign)[v * NW + lane] = reinterpret_cast<const uint32_t*>(b)[lane];
    if (lane == 0)
        reinterpret_cast<uint16_t*>(P.bscale)[v] = *reinterpret_cast<const uint16_t*>(b + kBinScaleOff);
    if (res != nullptr && P.nib != nullptr) {
        const uint16_t* r = reinterpret_cast<const uint16_t*>(res + v * kResRecBytes);
        uint8_t* nib = reinterpret_cast<uint8_t*>(P.nib);
        if constexpr (nib_by_bit(32 * NW)) {
            // lane b < head_dim / 8: record word b holds dims 8b .. 8b + 7 (nibble t = dim 8b + t);
            // the plane byte of (b, t) takes nibbles t (low) and t + 4 (high)
            if (lane < 4 * NW) {
                const uint32_t W = (uint32_t)r[2 * lane] | ((uint32_t)r[2 * lane + 1] << 16);
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    nib[nib_chunk_offset(v, nib_byte_chunk(32 * NW, lane, t), 32 * NW) +
                        nib_byte_index(32 * NW, lane, t)] =
                        (uint8_t)((((W >> (4 * t)) & 0xFu) | (((W >> (4 * t + 16)) & 0xFu) << 4)) ^ 0x88u);
            }
        } else {
            for (int i = lane; i < 8 * NW; i += 32)
                *reinterpret_cast<uint16_t*>(nib + nib_chunk_offset(v, i >> 3, 32 * NW) + 2 * (i & 7)) =
                    (uint16_t)(r[i] ^ 0x8888u);
        }
        if (lane == 0) reinterpret_cast<uint16_t*>(P.rscale)[v] = r[64];
    }
}

template <int NW>
__global__ void __launch_bounds__(kEncWarps * 32) k_planes_to_records(bc_kv_planes P, uint8_t* __restrict__ bin,
                                                                      uint8_t* __restrict__ res, int64_t n) {
    const int lane = threadIdx.x & 31;
    const int64_t v = (int64_t)blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (v >= n) return;
    uint32_t* b = reinterpret_cast<uint32_t*>(bin + v * kBinRecBytes);
    if (lane < 8) b[lane] = (lane < NW) ? reinterpret_cast<const uint32_t*>(P.sign)[v * NW + lane] : 0u;
    if (lane == 8) b[8] = (uint32_t)reinterpret_cast<const uint16_t*>(P.bscale)[v];
    if (res != nullptr && P.nib != nullptr) {
        uint16_t* r = reinterpret_cast<uint16_t*>(res + v * kResRecBytes);
        const uint8_t* nib = reinterpret_cast<const uint8_t*>(P.nib);
        if constexpr (nib_by_bit(32 * NW)) {
            // lane b < head_dim / 8 rebuilds record word b (dims 8b .. 8b + 7) from the
            // plane bytes of (b, t), t < 4
            if (lane < 4 * NW) {
                uint32_t W = 0;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t b = nib[nib_chunk_offset(v, nib_byte_chunk(32 * NW, lane, t), 32 * NW) +
                                           nib_byte_index(32 * NW, lane, t)] ^
                                       0x88u;
                    W |= ((b & 0xFu) << (4 * t)) | ((b >> 4) << (4 * t + 16));
                }
                r[2 * lane] = (uint16_t)W;
                r[2 * lane + 1] = (uint16_t)(W >> 16);
            }
            for (int i = 8 * NW + lane; i < 64; i += 32) r[i] = 0;  // record nibbles beyond head_dim
        } else {
            for (int i = lane; i < 64; i += 32)
                r[i] = (i < 8 * NW) ? (uint16_t)(*reinterpret_cast<const uint16_t*>(
                                                     nib + nib_chunk_offset(v, i >> 3, 32 * NW) + 2 * (i & 7)) ^
                                                 0x8888u)
                                    : (uint16_t)0;
        }
        if (lane == 0) r[64] = reinterpret_cast<const uint16_t*>(P.rscale)[v];
    }
}

}  // namespace bc

// ===========================================================================
// Entry points
// ===========================================================================
using namespace bc;

#define BC_DISPATCH_NW(d, KERNEL_CALL)               \
    switch ((d) / 32) {                              \
        case 1: { constexpr int NW = 1; KERNEL_CALL; break; } \
        case 2: { constexpr int NW = 2; KERNEL_CALL; break; } \
        case 3: { constexpr int NW = 3; KERNEL_CALL; break; } \
        case 4: { constexpr int NW = 4; KERNEL_CALL; break; } \
        case 5: { constexpr int NW = 5; KERNEL_CALL; break; } \
        case 6: { constexpr int NW = 6; KERNEL_CALL; break; } \
        case 7: { constexpr int NW = 7; KERNEL_CALL; break; } \
        case 8: { constexpr int NW = 8; KERNEL_CALL; break; } \
        default: return BC_ERR_HEAD_DIM;            \
    }

static inline unsigned enc_blocks(int64_t n) { return (unsigned)((n + kEncWarps - 1) / kEncWarps); }

template <int NW, int RES>
static int launch_lpv(const void* src, bc_kv_planes out, int64_t n, int seq_len, int64_t kv_stride, int head_dim,
                      int sms, cudaStream_t st) {
    constexpr int smem = LpvCfg<32 * NW>::SMEM_B;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaFuncSetAttribute(k_encode_planes_lpv<NW, RES>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        attr_set[dev] = true;
    }
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_encode_planes_lpv<NW, RES>, kLpvWarps * 32, smem);
    const int64_t batches = (n + 31) / 32;
    const int64_t want = (batches + kLpvWarps - 1) / kLpvWarps;
    const int64_t cap = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
    const unsigned blocks = (unsigned)(want < cap ? want : cap);
    k_encode_planes_lpv<NW, RES><<<blocks, kLpvWarps * 32, smem, st>>>((const __half*)src, out, seq_len, kv_stride,
                                                                        head_dim, n, bc_device_error_ptr());
    BC_LAUNCH_CHECK();
    return BC_OK;
}

template <int RES>
static int lpv_dispatch(const void* src, bc_kv_planes out, int64_t n, int seq_len, int64_t kv_stride, int head_dim,
                        int sms, cudaStream_t st) {
    switch (head_dim / 32) {
        case 1: return launch_lpv<1, RES>(src, out, n, seq_len, kv_stride, head_dim, sms, st);
        case 2: return launch_lpv<2, RES>(src, out, n, seq_len, kv_stride, head_dim, sms, st);
        case 3: return launch_lpv<3, RES>(src, out, n, seq_len, kv_stride, head_dim, sms, st);
        default: return launch_lpv<4, RES>(src, out, n, seq_len, kv_stride, head_dim, sms, st);
    }
}

static int encode_planes_lpv(const void* src, bc_kv_planes out, int64_t n, int seq_len, int64_t kv_stride,
                             int head_dim, int residual_mode, int sms, cudaStream_t st) {
    switch (residual_mode) {
        case BC_RES_NONE: return lpv_dispatch<BC_RES_NONE>(src, out, n, seq_len, kv_stride, head_dim, sms, st);
        case BC_RES_FP16_SCALE: return lpv_dispatch<BC_RES_FP16_SCALE>(src, out, n, seq_len, kv_stride, head_dim, sms, st);
        default: return lpv_dispatch<BC_RES_FP32_SCALE>(src, out, n, seq_len, kv_stride, head_dim, sms, st);
    }
}

extern "C" {

int64_t bc_sizeof_binary_vec(void) { return kBinRecBytes; }
int64_t bc_sizeof_residual_vec(void) { return kResRecBytes; }

const char* bc_status_string(int status) {
    switch (status) {
        case BC_OK: return "ok";
        case BC_ERR_HEAD_DIM: return "head_dim must be a multiple of 32 in [32, 256]";
        case BC_ERR_ARG: return "invalid argument (size, null pointer or mode)";
        case BC_ERR_ALIGN: return "pointer not 16-byte aligned or kv_stride not a multiple of 8";
        case BC_ERR_WORKSPACE: return "workspace too small";
        case BC_ERR_UNSUPPORTED: return "shape not supported by the compiled kernels";
        case BC_ERR_TOO_LARGE: return "size exceeds the fixed maximum of this entry point";
        default: break;
    }
    if (status >= BC_ERR_CUDA_BASE) return cudaGetErrorString((cudaError_t)(status - BC_ERR_CUDA_BASE));
    return "unknown status";
}

int bc_binary_encode(const void* src, void* out, int64_t n_vecs, int head_dim, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_vecs < 0) return BC_ERR_ARG;
    if (n_vecs == 0) return BC_OK;
    if (!src || !out) return BC_ERR_ARG;
    if (!bc_aligned(src, 2) || !bc_aligned(out, 4)) return BC_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    BC_DISPATCH_NW(head_dim, (k_binary_encode_rec<NW><<<enc_blocks(n_vecs), kEncWarps * 32, 0, st>>>(
                                  (const __half*)src, (uint8_t*)out, n_vecs, head_dim)));
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_residual_encode(const void* src, const void* bin, void* out, int64_t n_vecs, int head_dim, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_vecs < 0) return BC_ERR_ARG;
    if (n_vecs == 0) return BC_OK;
    if (!src || !bin || !out) return BC_ERR_ARG;
    if (!bc_aligned(src, 2) || !bc_aligned(bin, 4) || !bc_aligned(out, 2)) return BC_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    BC_DISPATCH_NW(head_dim, (k_residual_encode_rec<NW><<<enc_blocks(n_vecs), kEncWarps * 32, 0, st>>>(
                                  (const __half*)src, (const uint8_t*)bin, (uint8_t*)out, n_vecs, head_dim)));
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_online_encode_token(const void* kv, void* bin_cache, void* res_cache, int batch, int n_heads, int head_dim,
                           int current_len, int max_seq, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (batch < 0 || n_heads < 0 || max_seq <= 0 || current_len < 0) return BC_ERR_ARG;
    const int n_slots = batch * n_heads;
    if (n_slots == 0) return BC_OK;
    if (!kv || !bin_cache) return BC_ERR_ARG;
    if (!bc_aligned(kv, 2) || !bc_aligned(bin_cache, 4) || (res_cache && !bc_aligned(res_cache, 2)))
        return BC_ERR_ALIGN;
    const int write_slot = current_len % max_seq;
    cudaStream_t st = (cudaStream_t)stream;
    BC_DISPATCH_NW(head_dim, (k_online_encode_rec<NW><<<enc_blocks(n_slots), kEncWarps * 32, 0, st>>>(
                                  (const __half*)kv, (uint8_t*)bin_cache, (uint8_t*)res_cache, n_slots, head_dim,
                                  write_slot, max_seq)));
    BC_LAUNCH_CHECK();
    return BC_OK;
}

static int check_planes(const bc_kv_planes& P, bool need_res) {
    if (!P.sign || !P.bscale) return BC_ERR_ARG;
    if (need_res && (!P.nib || !P.rscale)) return BC_ERR_ARG;
    if (!bc_aligned(P.sign, 16) || !bc_aligned(P.bscale, 16)) return BC_ERR_ALIGN;
    if (need_res && (!bc_aligned(P.nib, 16) || !bc_aligned(P.rscale, 16))) return BC_ERR_ALIGN;
    return BC_OK;
}

int bc_encode_planes(const void* src, bc_kv_planes out, int n_slots, int seq_len, int64_t kv_stride, int head_dim,
                     int residual_mode, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_slots < 0 || seq_len < 0 || kv_stride < seq_len) return BC_ERR_ARG;
    if (residual_mode < BC_RES_NONE || residual_mode > BC_RES_FP32_SCALE) return BC_ERR_ARG;
    const int64_t n = (int64_t)n_slots * seq_len;
    if (n == 0) return BC_OK;
    if (!src) return BC_ERR_ARG;
    int rc = check_planes(out, residual_mode != BC_RES_NONE);
    if (rc) return rc;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t max_blocks = (int64_t)sms * 8;
    const int64_t want = (n + (int64_t)kEncWarps * kVecsPerWarp - 1) / ((int64_t)kEncWarps * kVecsPerWarp);
    const unsigned blocks = (unsigned)(want < max_blocks ? want : max_blocks);
    cudaStream_t st = (cudaStream_t)stream;
    if (head_dim <= 128 && bc_aligned(src, 16)) return encode_planes_lpv(src, out, n, seq_len, kv_stride, head_dim,
                                                                         residual_mode, sms, st);
    switch (residual_mode) {
        case BC_RES_NONE:
            BC_DISPATCH_NW(head_dim, (k_encode_planes<NW, BC_RES_NONE><<<blocks, kEncWarps * 32, 0, st>>>(
                                          (const __half*)src, out, n_slots, seq_len, kv_stride, head_dim)));
            break;
        case BC_RES_FP16_SCALE:
            BC_DISPATCH_NW(head_dim, (k_encode_planes<NW, BC_RES_FP16_SCALE><<<blocks, kEncWarps * 32, 0, st>>>(
                                          (const __half*)src, out, n_slots, seq_len, kv_stride, head_dim)));
            break;
        default:
            BC_DISPATCH_NW(head_dim, (k_encode_planes<NW, BC_RES_FP32_SCALE><<<blocks, kEncWarps * 32, 0, st>>>(
                                          (const __half*)src, out, n_slots, seq_len, kv_stride, head_dim)));
            break;
    }
    BC_LAUNCH_CHECK();
    return BC_OK;
}

static int append_kv(const void* k, const void* v, bc_kv_planes K, bc_kv_planes V, int n_slots, int head_dim,
                     int64_t kv_stride, int64_t pos, int residual_mode, bc_page_table pt, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_slots < 0 || pos < 0) return BC_ERR_ARG;
    if (!pt.pages && pos >= kv_stride) return BC_ERR_ARG;
    if (pt.pages && pos >= (int64_t)pt.max_pages * pt.page_size) return BC_ERR_ARG;
    if (residual_mode != BC_RES_NONE && residual_mode != BC_RES_FP32_SCALE && residual_mode != BC_RES_FP16_SCALE)
        return BC_ERR_ARG;
    if (n_slots == 0) return BC_OK;
    if (!k || !v) return BC_ERR_ARG;
    int rc = check_planes(K, residual_mode != BC_RES_NONE);
    if (rc) return rc;
    rc = check_planes(V, residual_mode != BC_RES_NONE);
    if (rc) return rc;
    unsigned int* err = pt.pages ? bc_device_error_ptr() : nullptr;
    cudaStream_t st = (cudaStream_t)stream;
    const unsigned blocks = enc_blocks(2 * (int64_t)n_slots);
    switch (residual_mode) {
        case BC_RES_NONE:
            BC_DISPATCH_NW(head_dim, (k_append_kv<NW, BC_RES_NONE><<<blocks, kEncWarps * 32, 0, st>>>(
                                          (const __half*)k, (const __half*)v, K, V, n_slots, head_dim, kv_stride, pos,
                                          pt, err)));
            break;
        case BC_RES_FP16_SCALE:
            BC_DISPATCH_NW(head_dim, (k_append_kv<NW, BC_RES_FP16_SCALE><<<blocks, kEncWarps * 32, 0, st>>>(
                                          (const __half*)k, (const __half*)v, K, V, n_slots, head_dim, kv_stride, pos,
                                          pt, err)));
            break;
        default:
            BC_DISPATCH_NW(head_dim, (k_append_kv<NW, BC_RES_FP32_SCALE><<<blocks, kEncWarps * 32, 0, st>>>(
                                          (const __half*)k, (const __half*)v, K, V, n_slots, head_dim, kv_stride, pos,
                                          pt, err)));
            break;
    }
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_append_kv(const void* k, const void* v, bc_kv_planes K, bc_kv_planes V, int n_slots, int head_dim,
                 int64_t kv_stride, int64_t pos, int residual_mode, void* stream) {
    return append_kv(k, v, K, V, n_slots, head_dim, kv_stride, pos, residual_mode, bc_page_table{}, stream);
}

int bc_append_kv_paged(const void* k, const void* v, bc_kv_planes K, bc_kv_planes V, bc_page_table pt, int n_slots,
                       int head_dim, int64_t pos, int residual_mode, void* stream) {
    if (!pt.pages || pt.page_size <= 0 || pt.page_size % 128 != 0 || pt.n_pages <= 0 || pt.max_pages <= 0)
        return BC_ERR_ARG;
    if (!bc_aligned(pt.pages, 4)) return BC_ERR_ALIGN;
    return append_kv(k, v, K, V, n_slots, head_dim, pt.page_size, pos, residual_mode, pt, stream);
}

int bc_records_to_planes(const void* binvec, const void* resvec, bc_kv_planes out, int64_t n_vecs, int head_dim,
                         void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_vecs < 0) return BC_ERR_ARG;
    if (n_vecs == 0) return BC_OK;
    if (!binvec || !out.sign || !out.bscale) return BC_ERR_ARG;
    if (resvec && (!out.nib || !out.rscale)) return BC_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    BC_DISPATCH_NW(head_dim, (k_records_to_planes<NW><<<enc_blocks(n_vecs), kEncWarps * 32, 0, st>>>(
                                  (const uint8_t*)binvec, (const uint8_t*)resvec, out, n_vecs)));
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_planes_to_records(bc_kv_planes in, void* binvec, void* resvec, int64_t n_vecs, int head_dim, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_vecs < 0) return BC_ERR_ARG;
    if (n_vecs == 0) return BC_OK;
    if (!binvec || !in.sign || !in.bscale) return BC_ERR_ARG;
    if (resvec && (!in.nib || !in.rscale)) return BC_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    BC_DISPATCH_NW(head_dim, (k_planes_to_records<NW><<<enc_blocks(n_vecs), kEncWarps * 32, 0, st>>>(
                                  in, (uint8_t*)binvec, (uint8_t*)resvec, n_vecs)));
    BC_LAUNCH_CHECK();
    return BC_OK;
}

}  // extern "C"
