// Fused split-K decode attention (binary and residual-compensated) over the
// plane cache layout, plus the reference-record variant.  sm_100a, SIMT:
// decode attention is GEMV-shaped (one query row per head) and HBM-bound.
//
// Arithmetic follows compensated_attention.cu:42-109 / binary_attention.cu:8-82
// of the reference:
//   score_s = (scale_q*scale_k*(2*popc(~(q_sign ^ k_sign)) - d)
//              + sum_i q_i*(n_i/7)*res_scale_k) / sqrt(d)
//   out     = sum_s softmax(score)_s * (sign_v*scale_v + (n_v/7)*res_scale_v)
// evaluated in one pass with an online softmax instead of the reference's two.
//
// Work decomposition.  A CTA of 256 threads owns one KV slot (batch, kv head),
// a contiguous key range (its split) and GC query heads of that slot's group.
// Tiles of T keys stream into a 4-stage shared-memory ring by 1-D TMA bulk
// copies (cp.async.bulk, no multicast) completing on mbarriers.  Each thread
// handles 32 consecutive dims of a key; QPK = d/32 threads form a key group
// and KPAR = 256/QPK groups walk the tile.  Every key group keeps its own
// online-softmax state; groups are merged once per CTA and splits once per
// slot by the last CTA to finish (atomic ticket), so one launch produces the
// final fp16 output.
//
// Scores.  Sign agreement: d - 2*popc(q_sign ^ k_sign) over the head.  The
// INT4 residual dot is exact integer arithmetic: each query element is
// quantised once to 16 bits (q ~= Q16 * qmax/32767) split into hi/lo bytes,
// nibbles are offset to unsigned (n+8) by one XOR and dotted with dp4a; the
// offset is removed with a precomputed 8*sum(Q16).
//
// Values.  For key weight w: sign part 2*a*b - a with a = w*scale_v, residual
// part c*(u - 8) with c = w*res_scale_v/7 and u = n+8.  Sign bits and nibbles
// are masked in place and used directly as fp32 denormal operands
// (pattern * 2^-149); packed fma.rn.f32x2 with power-of-two-rescaled
// coefficients turns them into exact multiples of 2^-64, and the constant
// parts sum_s (a_s + 8 c_s) are subtracted once at the end.
#include <mutex>

#include "common.cuh"

namespace bc {

__device__ unsigned int g_bc_device_error = 0;

constexpr int kDecThreads = 256;
constexpr int kStages = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLazy = 8.0f;   // rescale only when the running max grows by > 2^8
constexpr int kAccShift = 64;   // accumulators hold value * 2^-64

template <int D, int GC, bool COMP>
struct DecCfg {
    static constexpr int NWD = D / 32;            // sign words per key
    static constexpr int QPK = NWD;               // threads per key (32 dims each)
    static constexpr int KPAR = kDecThreads / QPK;
    static constexpr int KPT = 2;                 // keys per group per tile
    static constexpr int T = KPAR * KPT;          // keys per tile
    static constexpr int SIGN_B = T * D / 8;
    static constexpr int NIB_B = COMP ? T * D / 2 : 0;
    static constexpr int SC_B = T * 2;
    static constexpr int OFF_KSIGN = 0;
    static constexpr int OFF_KBS = OFF_KSIGN + SIGN_B;
    static constexpr int OFF_KNIB = OFF_KBS + SC_B;
    static constexpr int OFF_KRS = OFF_KNIB + NIB_B;
    static constexpr int OFF_VSIGN = OFF_KRS + (COMP ? SC_B : 0);
    static constexpr int OFF_VBS = OFF_VSIGN + SIGN_B;
    static constexpr int OFF_VNIB = OFF_VBS + SC_B;
    static constexpr int OFF_VRS = OFF_VNIB + NIB_B;
    static constexpr int STAGE_B = OFF_VRS + (COMP ? SC_B : 0);
    static constexpr int RING_B = kStages * STAGE_B;
    // merge scratch (reuses the ring): [warps][GC][D+2] floats
    static constexpr int MERGE_B = (kDecThreads / 32) * GC * (D + 2) * 4;
    static constexpr int BODY_B = RING_B > MERGE_B ? RING_B : MERGE_B;
    static constexpr int QF_OFF = BODY_B;                       // float q[GC][D]
    static constexpr int Q16_OFF = QF_OFF + GC * D * 4;         // int Q16[GC][D]
    static constexpr int QSIGN_OFF = Q16_OFF + GC * D * 4;      // uint32 [GC][8]
    static constexpr int QCONST_OFF = QSIGN_OFF + GC * 8 * 4;   // float bco, rco; int off8 -> [GC][4]
    static constexpr int BAR_OFF = QCONST_OFF + GC * 4 * 4;
    static constexpr int FLAG_OFF = BAR_OFF + kStages * 8;
    static constexpr int SMEM_B = FLAG_OFF + 16 + 128;  // + slack for aligning the base to 128 B
    static constexpr int MIN_BLOCKS = (GC == 1) ? 2 : 1;
};

struct DecodeArgs {
    const __half* q;    // [n_slots * group][d]
    bc_kv_planes K, V;  // planes, or record bases in .sign (bin) / .nib (res) for the record kernel
    __half* out;        // [n_slots * group][d] or null
    float* partial;     // [n_slots * group][d + 2] or null
    float* ws_part;     // [n_slots * group][n_splits][d + 2]
    unsigned* ws_cnt;   // [n_slots * n_hgroups]
    int n_slots, group, seq_len, n_splits, keys_per_split, n_hgroups;
    int64_t kv_stride;
    int head_dim;
};

// Per-thread query state for GC heads.
template <int GC>
struct QState {
    uint32_t sign[GC];
    uint32_t pk[GC][4][4];  // [head][nibble word][even hi, even lo, odd hi, odd lo]
    float bco[GC], rco[GC];
    int off8[GC];
};

template <int GC>
struct SoftState {
    float m[GC], l[GC], t[GC];
    f2 acc[GC][4][4];  // [head][nibble word w][j] -> dims (8w+j, 8w+4+j) of the thread's 32
};

// ---------------------------------------------------------------------------
// Query preparation (once per CTA).  scale_q is summed sequentially over the
// head as in compensated_attention.cu:65-67.
// ---------------------------------------------------------------------------
template <int D, int GC, bool COMP, typename Cfg>
__device__ __forceinline__ void prepare_query(const DecodeArgs& a, int slot, int hg, uint8_t* smem, QState<GC>& qs) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* qf = reinterpret_cast<float*>(smem + Cfg::QF_OFF);
    int* q16 = reinterpret_cast<int*>(smem + Cfg::Q16_OFF);
    uint32_t* qsign = reinterpret_cast<uint32_t*>(smem + Cfg::QSIGN_OFF);
    float* qc = reinterpret_cast<float*>(smem + Cfg::QCONST_OFF);
    const int64_t qbase = ((int64_t)slot * a.group + (int64_t)hg * GC) * D;
    for (int i = tid; i < GC * D; i += kDecThreads) qf[i] = __half2float(a.q[qbase + i]);
    __syncthreads();
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    if (warp < GC) {
        const int g = warp;
        float mx = 0.0f;
        for (int k = 0; k < D / 32; ++k) {
            const float v = qf[g * D + 32 * k + lane];
            const uint32_t w = __ballot_sync(0xffffffffu, v >= 0.0f);
            if (lane == k) qsign[g * 8 + k] = w;
            mx = fmaxf(mx, fabsf(v));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float qscale = mx > 0.0f ? 32767.0f / mx : 0.0f;
        int sum16 = 0;
        for (int k = 0; k < D / 32; ++k) {
            const int v = __float2int_rn(qf[g * D + 32 * k + lane] * qscale);
            q16[g * D + 32 * k + lane] = v;
            sum16 += v;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum16 += __shfl_xor_sync(0xffffffffu, sum16, off);
        if (lane == 0) {
            float sq = 0.0f;
            for (int i = 0; i < D; ++i) sq += fabsf(qf[g * D + i]);
            sq /= (float)D;
            qc[g * 4 + 0] = sq * inv_sqrt_d * kLog2e;
            qc[g * 4 + 1] = (mx / 32767.0f) * (1.0f / 7.0f) * inv_sqrt_d * kLog2e;
            reinterpret_cast<int*>(qc)[g * 4 + 2] = 8 * sum16;
        }
    }
    __syncthreads();
    const int qt = tid % Cfg::QPK;
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        qs.sign[g] = qsign[g * 8 + qt];
        qs.bco[g] = qc[g * 4 + 0];
        qs.rco[g] = qc[g * 4 + 1];
        qs.off8[g] = reinterpret_cast<const int*>(qc)[g * 4 + 2];
        if (COMP) {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                uint32_t eh = 0, el = 0, oh = 0, ol = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int de = g * D + 32 * qt + 8 * w + 2 * b;
                    const int ve = q16[de], vo = q16[de + 1];
                    eh |= ((uint32_t)(ve >> 8) & 0xFFu) << (8 * b);
                    el |= ((uint32_t)ve & 0xFFu) << (8 * b);
                    oh |= ((uint32_t)(vo >> 8) & 0xFFu) << (8 * b);
                    ol |= ((uint32_t)vo & 0xFFu) << (8 * b);
                }
                qs.pk[g][w][0] = eh;
                qs.pk[g][w][1] = el;
                qs.pk[g][w][2] = oh;
                qs.pk[g][w][3] = ol;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// One key: score for the GC heads (integer parts reduced across the QPK
// threads of the group), online softmax update, V accumulation for 32 dims.
// ---------------------------------------------------------------------------
template <int D, int GC, bool COMP>
__device__ __forceinline__ void consume_key(const QState<GC>& qs, SoftState<GC>& st, bool valid, uint32_t ks, float kbs,
                                            uint4 kn, float krs, uint32_t vs, float vbs, uint4 vn, float vrs) {
    constexpr int QPK = D / 32;
    float w_g[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        int pop = __popc(qs.sign[g] ^ ks);
        int dot = 0;
        if (COMP) {
            int hi = 0, lo = 0;
            const uint32_t nk[4] = {kn.x, kn.y, kn.z, kn.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const uint32_t nx = nk[w] ^ 0x88888888u;
                const uint32_t ue = nx & 0x0F0F0F0Fu;
                const uint32_t uo = (nx >> 4) & 0x0F0F0F0Fu;
                hi = dp4a_us(ue, qs.pk[g][w][0], hi);
                lo = dp4a_uu(ue, qs.pk[g][w][1], lo);
                hi = dp4a_us(uo, qs.pk[g][w][2], hi);
                lo = dp4a_uu(uo, qs.pk[g][w][3], lo);
            }
            dot = hi * 256 + lo;
        }
#pragma unroll
        for (int off = 1; off < QPK; off <<= 1) {
            pop += __shfl_xor_sync(0xffffffffu, pop, off);
            if (COMP) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        }
        // Shuffles above run on every lane; everything below is per key group and
        // skipped for keys past the end of the range.
        float s2 = qs.bco[g] * kbs * (float)(D - 2 * pop);
        if (COMP) s2 = fmaf(qs.rco[g] * krs, (float)(dot - qs.off8[g]), s2);
        if (!valid) s2 = -INFINITY;
        if (s2 > st.m[g] + kLazy) {
            const float alpha = fast_exp2(st.m[g] - s2);
            st.m[g] = s2;
            st.l[g] *= alpha;
            st.t[g] *= alpha;
            const f2 al = {alpha, alpha};
#pragma unroll
            for (int w = 0; w < 4; ++w)
#pragma unroll
                for (int j = 0; j < 4; ++j) fmul2(st.acc[g][w][j], al);
        }
        const float wt = valid ? fast_exp2(s2 - st.m[g]) : 0.0f;
        st.l[g] += wt;
        w_g[g] = wt;
    }
    if (!valid) return;
    // V accumulation
    const uint32_t nv[4] = {vn.x, vn.y, vn.z, vn.w};
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        const float av = w_g[g] * vbs;
        const float A0 = 2.0f * av * exp2i(149 - kAccShift);
        float C0 = 0.0f;
        if (COMP) {
            const float cv = w_g[g] * vrs * (1.0f / 7.0f);
            C0 = cv * exp2i(149 - kAccShift);
            st.t[g] += av + 8.0f * cv;
        } else {
            st.t[g] += av;
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint32_t sw = vs >> (8 * w);
            const uint32_t sw4 = vs >> (8 * w + 4);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float Aj = A0 * exp2i(-j);
                const f2 y = {bits_f(sw & (1u << j)), bits_f(sw4 & (1u << j))};
                ffma2(st.acc[g][w][j], f2{Aj, Aj}, y);
            }
            if (COMP) {
                const uint32_t nx = nv[w] ^ 0x88888888u;
                const uint32_t nh = nx >> 16;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float Cj = C0 * exp2i(-4 * j);
                    const f2 x = {bits_f(nx & (0xFu << (4 * j))), bits_f(nh & (0xFu << (4 * j)))};
                    ffma2(st.acc[g][w][j], f2{Cj, Cj}, x);
                }
            }
        }
    }
}

// Convert accumulator pair (w, j) to true unnormalised value of dims (8w+j, 8w+4+j).
__device__ __forceinline__ float acc_true(float acc_scaled, float t) { return acc_scaled * exp2i(kAccShift) - t; }

// ---------------------------------------------------------------------------
// Merge all key groups of the CTA, then (split-K) publish a partial and let the
// last CTA of the slot combine and write the outputs.
// ---------------------------------------------------------------------------
template <int D, int GC, typename Cfg>
__device__ __forceinline__ void finish_cta(const DecodeArgs& a, int slot, int hg, int split, uint8_t* smem,
                                           SoftState<GC>& st) {
    constexpr int QPK = Cfg::QPK;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, qt = tid % QPK;
    // per-thread true values for its 32 dims, ordered by dim
    float o[GC][32];
#pragma unroll
    for (int g = 0; g < GC; ++g)
#pragma unroll
        for (int w = 0; w < 4; ++w)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                o[g][8 * w + j] = acc_true(st.acc[g][w][j].x, st.t[g]);
                o[g][8 * w + 4 + j] = acc_true(st.acc[g][w][j].y, st.t[g]);
            }
    // warp-level merge across key groups (lanes differing in bits >= log2(QPK))
#pragma unroll
    for (int off = QPK; off < 32; off <<= 1) {
#pragma unroll
        for (int g = 0; g < GC; ++g) {
            const float mp = __shfl_xor_sync(0xffffffffu, st.m[g], off);
            const float lp = __shfl_xor_sync(0xffffffffu, st.l[g], off);
            const float M = fmaxf(st.m[g], mp);
            const float fa = (st.m[g] == -INFINITY) ? 0.0f : fast_exp2(st.m[g] - M);
            const float fb = (mp == -INFINITY) ? 0.0f : fast_exp2(mp - M);
            st.l[g] = st.l[g] * fa + lp * fb;
            st.m[g] = M;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float op = __shfl_xor_sync(0xffffffffu, o[g][i], off);
                o[g][i] = o[g][i] * fa + op * fb;
            }
        }
    }
    __syncthreads();  // ring no longer in use
    float* mg = reinterpret_cast<float*>(smem);  // [warps][GC][D+2]
    if (lane < QPK) {
#pragma unroll
        for (int g = 0; g < GC; ++g) {
            float* rec = mg + ((size_t)warp * GC + g) * (D + 2);
            if (lane == 0) {
                rec[0] = st.m[g];
                rec[1] = st.l[g];
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) rec[2 + 32 * qt + i] = o[g][i];
        }
    }
    __syncthreads();
    constexpr int NWARP = kDecThreads / 32;
    // cross-warp merge: thread handles (g, dim)
    const bool single = (a.n_splits == 1);
    const int64_t head0 = (int64_t)slot * a.group + (int64_t)hg * GC;
    for (int idx = tid; idx < GC * D; idx += kDecThreads) {
        const int g = idx / D, i = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) M = fmaxf(M, mg[((size_t)w * GC + g) * (D + 2)]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
            const float* rec = mg + ((size_t)w * GC + g) * (D + 2);
            const float f = (rec[0] == -INFINITY) ? 0.0f : fast_exp2(rec[0] - M);
            L += rec[1] * f;
            O += rec[2 + i] * f;
        }
        const int64_t h = head0 + g;
        if (single) {
            if (a.out) a.out[h * D + i] = __float2half((L > 0.0f) ? O * (1.0f / L) : 0.0f);
            if (a.partial) {
                float* p = a.partial + h * (D + 2);
                if (i == 0) {
                    p[0] = M * kLn2;
                    p[1] = L;
                }
                p[2 + i] = O;
            }
        } else {
            float* p = a.ws_part + (h * a.n_splits + split) * (D + 2);
            if (i == 0) {
                p[0] = M;
                p[1] = L;
            }
            p[2 + i] = O;
        }
    }
    if (single) return;
    // ticket: the last CTA of this (slot, head group) combines the splits
    __shared__ unsigned s_last;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&a.ws_cnt[(int64_t)slot * a.n_hgroups + hg], 1u);
        s_last = (prev == (unsigned)(a.n_splits - 1)) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int idx = tid; idx < GC * D; idx += kDecThreads) {
        const int g = idx / D, i = idx % D;
        const int64_t h = head0 + g;
        const float* base = a.ws_part + h * a.n_splits * (D + 2);
        float M = -INFINITY;
        for (int j = 0; j < a.n_splits; ++j) M = fmaxf(M, __ldcg(base + (size_t)j * (D + 2)));
        float L = 0.0f, O = 0.0f;
        for (int j = 0; j < a.n_splits; ++j) {
            const float mj = __ldcg(base + (size_t)j * (D + 2));
            const float f = (mj == -INFINITY) ? 0.0f : fast_exp2(mj - M);
            L += __ldcg(base + (size_t)j * (D + 2) + 1) * f;
            O += __ldcg(base + (size_t)j * (D + 2) + 2 + i) * f;
        }
        if (a.out) a.out[h * D + i] = __float2half((L > 0.0f) ? O * (1.0f / L) : 0.0f);
        if (a.partial) {
            float* p = a.partial + h * (D + 2);
            if (i == 0) {
                p[0] = M * kLn2;
                p[1] = L;
            }
            p[2 + i] = O;
        }
    }
    if (tid == 0) a.ws_cnt[(int64_t)slot * a.n_hgroups + hg] = 0u;  // leave the workspace zeroed
}

template <int GC>
__device__ __forceinline__ void init_soft(SoftState<GC>& st) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        st.m[g] = -INFINITY;
        st.l[g] = 0.0f;
        st.t[g] = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w)
#pragma unroll
            for (int j = 0; j < 4; ++j) st.acc[g][w][j] = f2{0.0f, 0.0f};
    }
}

// ---------------------------------------------------------------------------
// Plane-layout kernel (TMA ring)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 127) & ~uintptr_t(127));
}

template <int D, int GC, bool COMP>
__global__ void __launch_bounds__(kDecThreads, DecCfg<D, GC, COMP>::MIN_BLOCKS)
    k_decode_planes(const DecodeArgs a) {
    using Cfg = DecCfg<D, GC, COMP>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = aligned_smem(smem_raw);
    const int tid = threadIdx.x;
    const int cta = blockIdx.x;
    const int split = cta % a.n_splits;
    const int rest = cta / a.n_splits;
    const int hg = rest % a.n_hgroups;
    const int slot = rest / a.n_hgroups;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);

    const int s_begin = split * a.keys_per_split;
    const int s_end = min(a.seq_len, s_begin + a.keys_per_split);
    const int n_keys = max(0, s_end - s_begin);
    const int n_tiles = (n_keys + Cfg::T - 1) / Cfg::T;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int64_t row_base = (int64_t)slot * a.kv_stride + s_begin;
    auto issue = [&](int tile, int stage) {
        const int k0 = tile * Cfg::T;
        const int nk = min(Cfg::T, n_keys - k0);
        const int nk8 = (nk + 7) & ~7;
        const int64_t row = row_base + k0;
        uint8_t* sb = smem + stage * Cfg::STAGE_B;
        const uint32_t sign_b = nk8 * (D / 8), sc_b = nk8 * 2, nib_b = nk8 * (D / 2);
        const uint32_t total = 2 * (sign_b + sc_b + (COMP ? nib_b + sc_b : 0));
        mbar_arrive_expect_tx(&bars[stage], total);
        bulk_g2s(sb + Cfg::OFF_KSIGN, (const uint8_t*)a.K.sign + row * (D / 8), sign_b, &bars[stage]);
        bulk_g2s(sb + Cfg::OFF_KBS, (const uint8_t*)a.K.bscale + row * 2, sc_b, &bars[stage]);
        bulk_g2s(sb + Cfg::OFF_VSIGN, (const uint8_t*)a.V.sign + row * (D / 8), sign_b, &bars[stage]);
        bulk_g2s(sb + Cfg::OFF_VBS, (const uint8_t*)a.V.bscale + row * 2, sc_b, &bars[stage]);
        if (COMP) {
            bulk_g2s(sb + Cfg::OFF_KNIB, (const uint8_t*)a.K.nib + row * (D / 2), nib_b, &bars[stage]);
            bulk_g2s(sb + Cfg::OFF_KRS, (const uint8_t*)a.K.rscale + row * 2, sc_b, &bars[stage]);
            bulk_g2s(sb + Cfg::OFF_VNIB, (const uint8_t*)a.V.nib + row * (D / 2), nib_b, &bars[stage]);
            bulk_g2s(sb + Cfg::OFF_VRS, (const uint8_t*)a.V.rscale + row * 2, sc_b, &bars[stage]);
        }
    };
    if (tid == 0) {
        const int pre = min(kStages - 1, n_tiles);
        for (int t = 0; t < pre; ++t) issue(t, t);
    }

    QState<GC> qs;
    prepare_query<D, GC, COMP, Cfg>(a, slot, hg, smem, qs);
    SoftState<GC> st;
    init_soft<GC>(st);

    const int grp = tid / Cfg::QPK, qt = tid % Cfg::QPK;
    for (int it = 0; it < n_tiles; ++it) {
        const int stage = it % kStages;
        const uint32_t parity = (uint32_t)(it / kStages) & 1u;
        if (tid == 0 && it + kStages - 1 < n_tiles) {
            fence_proxy_async_smem();
            issue(it + kStages - 1, (it + kStages - 1) % kStages);
        }
        const bool ok = mbar_wait_bounded(&bars[stage], parity);
        if (ok) {
            const uint8_t* sb = smem + stage * Cfg::STAGE_B;
            const int nk = min(Cfg::T, n_keys - it * Cfg::T);
#pragma unroll
            for (int kk = 0; kk < Cfg::KPT; ++kk) {
                const int key = grp + kk * Cfg::KPAR;
                {
                    const uint32_t ks = reinterpret_cast<const uint32_t*>(sb + Cfg::OFF_KSIGN)[key * Cfg::NWD + qt];
                    const float kbs = __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_KBS)[key]);
                    const uint32_t vs = reinterpret_cast<const uint32_t*>(sb + Cfg::OFF_VSIGN)[key * Cfg::NWD + qt];
                    const float vbs = __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_VBS)[key]);
                    uint4 kn = make_uint4(0, 0, 0, 0), vn = make_uint4(0, 0, 0, 0);
                    float krs = 0.0f, vrs = 0.0f;
                    if (COMP) {
                        kn = reinterpret_cast<const uint4*>(sb + Cfg::OFF_KNIB)[key * Cfg::NWD + qt];
                        krs = __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_KRS)[key]);
                        vn = reinterpret_cast<const uint4*>(sb + Cfg::OFF_VNIB)[key * Cfg::NWD + qt];
                        vrs = __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_VRS)[key]);
                    }
                    consume_key<D, GC, COMP>(qs, st, key < nk, ks, kbs, kn, krs, vs, vbs, vn, vrs);
                }
            }
        }
        if (__syncthreads_or(!ok)) {
            // A copy never landed: report, drain what is still in flight (bounded), leave.
            if (tid == 0) {
                raise_device_error(&g_bc_device_error, BC_DEVERR_TIMEOUT);
                for (int t = it; t < min(n_tiles, it + kStages); ++t)
                    mbar_wait_bounded(&bars[t % kStages], (uint32_t)(t / kStages) & 1u);
            }
            return;
        }
    }
    finish_cta<D, GC, Cfg>(a, slot, hg, split, smem, st);
}

// ---------------------------------------------------------------------------
// Reference-record kernel: same math, fields read straight from BinaryVec
// (36 B) / ResidualVec (130 B, 2-byte aligned) arrays.  K, V record bases are
// passed in .sign (BinaryVec*) and .nib (ResidualVec*), kv_stride = seq_len.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 load_res_nibbles16(const uint8_t* p) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
    uint4 r;
    r.x = (uint32_t)__ldg(h + 0) | ((uint32_t)__ldg(h + 1) << 16);
    r.y = (uint32_t)__ldg(h + 2) | ((uint32_t)__ldg(h + 3) << 16);
    r.z = (uint32_t)__ldg(h + 4) | ((uint32_t)__ldg(h + 5) << 16);
    r.w = (uint32_t)__ldg(h + 6) | ((uint32_t)__ldg(h + 7) << 16);
    return r;
}

template <int D, int GC, bool COMP>
__global__ void __launch_bounds__(kDecThreads, DecCfg<D, GC, COMP>::MIN_BLOCKS)
    k_decode_records(const DecodeArgs a) {
    using Cfg = DecCfg<D, GC, COMP>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = aligned_smem(smem_raw);
    const int tid = threadIdx.x;
    const int cta = blockIdx.x;
    const int split = cta % a.n_splits;
    const int rest = cta / a.n_splits;
    const int hg = rest % a.n_hgroups;
    const int slot = rest / a.n_hgroups;
    const int s_begin = split * a.keys_per_split;
    const int s_end = min(a.seq_len, s_begin + a.keys_per_split);

    QState<GC> qs;
    prepare_query<D, GC, COMP, Cfg>(a, slot, hg, smem, qs);
    SoftState<GC> st;
    init_soft<GC>(st);

    const int grp = tid / Cfg::QPK, qt = tid % Cfg::QPK;
    const uint8_t* kb = (const uint8_t*)a.K.sign;
    const uint8_t* kr = (const uint8_t*)a.K.nib;
    const uint8_t* vb = (const uint8_t*)a.V.sign;
    const uint8_t* vr = (const uint8_t*)a.V.nib;
    const int64_t base = (int64_t)slot * a.kv_stride;
    const int n_keys = max(0, s_end - s_begin);
    const int trips = (n_keys + Cfg::KPAR - 1) / Cfg::KPAR;
    for (int tr = 0; tr < trips; ++tr) {
        const int s = s_begin + grp + tr * Cfg::KPAR;
        const bool valid = s < s_end;
        const int64_t rec = base + (valid ? s : s_begin);
        const uint8_t* kbr = kb + rec * kBinRecBytes;
        const uint8_t* vbr = vb + rec * kBinRecBytes;
        const uint32_t ks = __ldg(reinterpret_cast<const uint32_t*>(kbr) + qt);
        const float kbs = __half2float(__ldg(reinterpret_cast<const __half*>(kbr + kBinScaleOff)));
        const uint32_t vs = __ldg(reinterpret_cast<const uint32_t*>(vbr) + qt);
        const float vbs = __half2float(__ldg(reinterpret_cast<const __half*>(vbr + kBinScaleOff)));
        uint4 kn = make_uint4(0, 0, 0, 0), vn = make_uint4(0, 0, 0, 0);
        float krs = 0.0f, vrs = 0.0f;
        if (COMP) {
            const uint8_t* krr = kr + rec * kResRecBytes;
            const uint8_t* vrr = vr + rec * kResRecBytes;
            kn = load_res_nibbles16(krr + 16 * qt);
            krs = __half2float(__ldg(reinterpret_cast<const __half*>(krr + kResScaleOff)));
            vn = load_res_nibbles16(vrr + 16 * qt);
            vrs = __half2float(__ldg(reinterpret_cast<const __half*>(vrr + kResScaleOff)));
        }
        consume_key<D, GC, COMP>(qs, st, valid, ks, kbs, kn, krs, vs, vbs, vn, vrs);
    }
    finish_cta<D, GC, Cfg>(a, slot, hg, split, smem, st);
}

// ---------------------------------------------------------------------------
// Small kernels: log-sum-exp merge of partial triples, xnor popcount scores.
// ---------------------------------------------------------------------------
__global__ void k_lse_merge(const float* __restrict__ parts, int n_parts, int64_t n_heads, int d,
                            __half* __restrict__ out) {
    const int64_t h = blockIdx.x;
    float M = -INFINITY;
    for (int p = 0; p < n_parts; ++p) {
        const float* r = parts + ((int64_t)p * n_heads + h) * (d + 2);
        if (r[1] > 0.0f) M = fmaxf(M, r[0]);
    }
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        float L = 0.0f, O = 0.0f;
        for (int p = 0; p < n_parts; ++p) {
            const float* r = parts + ((int64_t)p * n_heads + h) * (d + 2);
            if (!(r[1] > 0.0f)) continue;
            const float f = __expf(r[0] - M);
            L += r[1] * f;
            O += r[2 + i] * f;
        }
        out[h * d + i] = __float2half((L > 0.0f) ? O / L : 0.0f);
    }
}

__global__ void k_xnor_popcount(const __half* __restrict__ q, const uint32_t* __restrict__ ksign,
                                int32_t* __restrict__ out, int n_heads, int group, int seq_len, int64_t kv_stride,
                                int d) {
    const int h = blockIdx.y;
    const int nw = d / 32;
    __shared__ uint32_t qs[8];
    if (threadIdx.x < 32) {
        for (int k = 0; k < nw; ++k) {
            const uint32_t w = __ballot_sync(0xffffffffu, __half2float(q[(int64_t)h * d + 32 * k + threadIdx.x]) >= 0.0f);
            if (threadIdx.x == 0) qs[k] = w;
        }
    }
    __syncthreads();
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= seq_len) return;
    const uint32_t* kr = ksign + ((int64_t)(h / group) * kv_stride + s) * nw;
    int p = 0;
    for (int k = 0; k < nw; ++k) p += __popc(~(qs[k] ^ kr[k]));
    out[(int64_t)h * seq_len + s] = p;
}

}  // namespace bc

// ===========================================================================
// Host side: split planning and entry points
// ===========================================================================
using namespace bc;

namespace {

constexpr int kMaxCtasPlan = 640;  // device-independent bound used for workspace sizing

struct Plan {
    int n_splits, keys_per_split, n_hgroups, gc, tile;
};

int tile_keys(int d) { return 2 * (kDecThreads / (d / 32)); }

int heads_per_cta(int group) { return group >= 2 ? 2 : 1; }

// Choose the split count so that all CTAs fit in one resident wave when the
// slots alone cannot fill the GPU (avoids a ragged second wave).
Plan make_plan(int n_slots, int group, int seq_len, int d, int capacity) {
    Plan p;
    p.gc = heads_per_cta(group);
    p.n_hgroups = group / p.gc;
    p.tile = tile_keys(d);
    const int n_tiles = max(1, (seq_len + p.tile - 1) / p.tile);
    const int64_t units = (int64_t)n_slots * p.n_hgroups;
    int splits = 1;
    if (units < capacity) splits = (int)(capacity / units);
    splits = max(1, min(splits, n_tiles));
    const int tiles_per_split = (n_tiles + splits - 1) / splits;
    p.keys_per_split = tiles_per_split * p.tile;
    p.n_splits = max(1, (max(seq_len, 1) + p.keys_per_split - 1) / p.keys_per_split);
    return p;
}

size_t ws_bytes_for(int n_slots, int group, int n_splits, int d, int n_hgroups) {
    const size_t part = (size_t)n_slots * group * n_splits * (d + 2) * sizeof(float);
    const size_t cnt = (size_t)n_slots * n_hgroups * sizeof(unsigned);
    return ((part + 255) & ~(size_t)255) + ((cnt + 255) & ~(size_t)255);
}

int max_plan_splits(int n_slots, int group, int seq_len, int d) {
    return make_plan(n_slots, group, seq_len, d, kMaxCtasPlan).n_splits;
}

template <int D, int GC, bool COMP>
int launch_decode(const DecodeArgs& a, bool records, cudaStream_t st) {
    using Cfg = DecCfg<D, GC, COMP>;
    const unsigned grid = (unsigned)((int64_t)a.n_slots * a.n_hgroups * a.n_splits);
    if (grid == 0) return BC_OK;
    if (records)
        k_decode_records<D, GC, COMP><<<grid, kDecThreads, Cfg::SMEM_B, st>>>(a);
    else
        k_decode_planes<D, GC, COMP><<<grid, kDecThreads, Cfg::SMEM_B, st>>>(a);
    BC_LAUNCH_CHECK();
    return BC_OK;
}

// Sets the dynamic shared-memory limit of both kernel variants on the current
// device (once per device) and returns the resident-CTA capacity of the GPU.
template <int D, int GC, bool COMP>
int capacity_of(bool records) {
    using Cfg = DecCfg<D, GC, COMP>;
    constexpr int kMaxDev = 64;
    static int cap[2][kMaxDev] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDev && cap[records][dev] > 0) return cap[records][dev];
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (records) {
        cudaFuncSetAttribute(k_decode_records<D, GC, COMP>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_B);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_records<D, GC, COMP>, kDecThreads,
                                                      Cfg::SMEM_B);
    } else {
        cudaFuncSetAttribute(k_decode_planes<D, GC, COMP>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_B);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_planes<D, GC, COMP>, kDecThreads,
                                                      Cfg::SMEM_B);
    }
    const int c = sms * max(1, per_sm);
    if (dev >= 0 && dev < kMaxDev) cap[records][dev] = c;
    return c;
}

template <int D, int GC, bool COMP>
int run_decode_t(DecodeArgs a, bool records, void* ws, size_t ws_bytes, cudaStream_t st) {
    const int cap = min(capacity_of<D, GC, COMP>(records), kMaxCtasPlan);
    Plan p = make_plan(a.n_slots, a.group, a.seq_len, D, cap);
    a.n_splits = p.n_splits;
    a.keys_per_split = p.keys_per_split;
    a.n_hgroups = p.n_hgroups;
    if (p.n_splits > 1) {
        const size_t need = ws_bytes_for(a.n_slots, a.group, p.n_splits, D, p.n_hgroups);
        if (ws == nullptr || ws_bytes < need) return BC_ERR_WORKSPACE;
        // Ticket counters first, at a fixed offset: calls of any shape find them
        // zero (every completed call resets its own); partials follow and are
        // always written before they are read.
        const size_t cnt = (size_t)a.n_slots * p.n_hgroups * sizeof(unsigned);
        a.ws_cnt = reinterpret_cast<unsigned*>(ws);
        a.ws_part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + ((cnt + 255) & ~(size_t)255));
    } else {
        a.ws_part = nullptr;
        a.ws_cnt = nullptr;
    }
    return launch_decode<D, GC, COMP>(a, records, st);
}

template <int D>
int run_decode_d(const DecodeArgs& a, bool comp, bool records, void* ws, size_t wsb, cudaStream_t st) {
    const int gc = heads_per_cta(a.group);
    if (gc == 1) return comp ? run_decode_t<D, 1, true>(a, records, ws, wsb, st) : run_decode_t<D, 1, false>(a, records, ws, wsb, st);
    return comp ? run_decode_t<D, 2, true>(a, records, ws, wsb, st) : run_decode_t<D, 2, false>(a, records, ws, wsb, st);
}

int run_decode(const DecodeArgs& a, bool comp, bool records, void* ws, size_t wsb, cudaStream_t st) {
    switch (a.head_dim) {
        case 32: return run_decode_d<32>(a, comp, records, ws, wsb, st);
        case 64: return run_decode_d<64>(a, comp, records, ws, wsb, st);
        case 128: return run_decode_d<128>(a, comp, records, ws, wsb, st);
        case 256: return run_decode_d<256>(a, comp, records, ws, wsb, st);
        default: return BC_ERR_UNSUPPORTED;
    }
}

bool valid_group(int g) { return g == 1 || g == 2 || g == 4 || g == 8; }

}  // namespace

extern "C" {

unsigned int bc_get_device_error(int clear) {
    unsigned int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xFFFFFFFFu;
    if (cudaMemcpyFromSymbol(&v, g_bc_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear) {
        unsigned int z = 0;
        cudaMemcpyToSymbol(g_bc_device_error, &z, sizeof(z));
    }
    return v;
}

size_t bc_decode_workspace_bytes(int n_slots, int group, int seq_len, int head_dim) {
    if (n_slots <= 0 || !valid_group(group) || seq_len < 0 || !bc_valid_head_dim(head_dim)) return 0;
    const int gc = heads_per_cta(group);
    const int s = max_plan_splits(n_slots, group, seq_len, head_dim);
    return ws_bytes_for(n_slots, group, s, head_dim, group / gc);
}

int bc_decode_attention(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial, int n_slots,
                        int group, int seq_len, int64_t kv_stride, int head_dim, int mode, void* workspace,
                        size_t workspace_bytes, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) return BC_ERR_UNSUPPORTED;
    if (!valid_group(group)) return BC_ERR_UNSUPPORTED;
    if (n_slots < 0 || seq_len < 0 || kv_stride < seq_len) return BC_ERR_ARG;
    if (mode != BC_MODE_BINARY && mode != BC_MODE_COMPENSATED) return BC_ERR_ARG;
    if (n_slots == 0) return BC_OK;
    if (!q || (!out && !partial)) return BC_ERR_ARG;
    if (kv_stride % 8 != 0) return BC_ERR_ALIGN;
    const bool comp = mode == BC_MODE_COMPENSATED;
    if (!K.sign || !K.bscale || !V.sign || !V.bscale) return BC_ERR_ARG;
    if (comp && (!K.nib || !K.rscale || !V.nib || !V.rscale)) return BC_ERR_ARG;
    const void* ptrs[8] = {K.sign, K.bscale, V.sign, V.bscale, K.nib, K.rscale, V.nib, V.rscale};
    for (int i = 0; i < (comp ? 8 : 4); ++i)
        if (!bc_aligned(ptrs[i], 16)) return BC_ERR_ALIGN;
    if (!bc_aligned(q, 2) || (out && !bc_aligned(out, 2)) || (partial && !bc_aligned(partial, 4))) return BC_ERR_ALIGN;
    DecodeArgs a{};
    a.q = (const __half*)q;
    a.K = K;
    a.V = V;
    a.out = (__half*)out;
    a.partial = partial;
    a.n_slots = n_slots;
    a.group = group;
    a.seq_len = seq_len;
    a.kv_stride = kv_stride;
    a.head_dim = head_dim;
    return run_decode(a, comp, false, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t bc_attention_workspace_bytes(int batch, int n_heads, int seq_len, int head_dim) {
    if (batch <= 0 || n_heads <= 0) return 0;
    return bc_decode_workspace_bytes(batch * n_heads, 1, seq_len, head_dim);
}

static int record_attention(const void* q, const void* kb, const void* kr, const void* vb, const void* vr, void* out,
                            int batch, int n_heads, int seq_len, int head_dim, bool comp, void* ws, size_t wsb,
                            void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) return BC_ERR_UNSUPPORTED;
    if (batch < 0 || n_heads < 0 || seq_len < 0) return BC_ERR_ARG;
    const int n = batch * n_heads;
    if (n == 0) return BC_OK;
    if (!q || !kb || !vb || !out || (comp && (!kr || !vr))) return BC_ERR_ARG;
    if (!bc_aligned(kb, 4) || !bc_aligned(vb, 4) || (comp && (!bc_aligned(kr, 2) || !bc_aligned(vr, 2))))
        return BC_ERR_ALIGN;
    DecodeArgs a{};
    a.q = (const __half*)q;
    a.K.sign = const_cast<void*>(kb);
    a.K.nib = const_cast<void*>(kr);
    a.V.sign = const_cast<void*>(vb);
    a.V.nib = const_cast<void*>(vr);
    a.out = (__half*)out;
    a.partial = nullptr;
    a.n_slots = n;
    a.group = 1;
    a.seq_len = seq_len;
    a.kv_stride = seq_len;
    a.head_dim = head_dim;
    return run_decode(a, comp, true, ws, wsb, (cudaStream_t)stream);
}

int bc_binary_attention(const void* q, const void* k_bin, const void* v_bin, void* out, int batch, int n_heads,
                        int seq_len, int head_dim, void* workspace, size_t workspace_bytes, void* stream) {
    return record_attention(q, k_bin, nullptr, v_bin, nullptr, out, batch, n_heads, seq_len, head_dim, false,
                            workspace, workspace_bytes, stream);
}

int bc_compensated_attention(const void* q, const void* k_bin, const void* k_res, const void* v_bin,
                             const void* v_res, void* out, int batch, int n_heads, int seq_len, int head_dim,
                             void* workspace, size_t workspace_bytes, void* stream) {
    return record_attention(q, k_bin, k_res, v_bin, v_res, out, batch, n_heads, seq_len, head_dim, true, workspace,
                            workspace_bytes, stream);
}

int bc_lse_merge(const float* parts, int n_parts, int64_t n_heads, int head_dim, void* out, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_parts <= 0 || n_heads < 0) return BC_ERR_ARG;
    if (n_heads == 0) return BC_OK;
    if (!parts || !out) return BC_ERR_ARG;
    k_lse_merge<<<(unsigned)n_heads, 128, 0, (cudaStream_t)stream>>>(parts, n_parts, n_heads, head_dim,
                                                                       (__half*)out);
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_xnor_popcount(const void* q, const void* k_sign, int32_t* out, int n_slots, int group, int seq_len,
                     int64_t kv_stride, int head_dim, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_slots < 0 || group <= 0 || seq_len < 0 || kv_stride < seq_len) return BC_ERR_ARG;
    const int n_heads = n_slots * group;
    if (n_heads == 0 || seq_len == 0) return BC_OK;
    if (!q || !k_sign || !out) return BC_ERR_ARG;
    dim3 grid((seq_len + 255) / 256, n_heads);
    k_xnor_popcount<<<grid, 256, 0, (cudaStream_t)stream>>>((const __half*)q, (const uint32_t*)k_sign, out, n_heads,
                                                            group, seq_len, kv_stride, head_dim);
    BC_LAUNCH_CHECK();
    return BC_OK;
}

}  // extern "C"

// ===========================================================================
// Allocation-free decode attention.
//
// Some callers cannot allocate device memory at the point where they run
// attention: an inference server that reserves all of its GPU memory up
// front and forbids allocation in the decode loop, or a plugin whose host
// framework owns every device buffer and hands it only inputs and outputs.
// They get this one extra entry point.  Its split-K scratch (ticket counters
// and partial results) lives in a fixed array inside the library instead of
// a caller workspace; every GPU that loads the library holds the array until
// the process exits.
// ===========================================================================
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_bc_static_scratch[kStaticScratchBytes];

constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_scratch_addr[kStaticMaxDevices] = {};

// Device address of the array on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
int static_scratch_address(void** addr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    if (dev < 0 || dev >= kStaticMaxDevices) return BC_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_bc_static_scratch);
        if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
        g_static_scratch_addr[dev] = p;
    }
    *addr = g_static_scratch_addr[dev];
    return BC_OK;
}

}  // namespace

extern "C" {

size_t bc_decode_noalloc_max_scratch_bytes(void) { return kStaticScratchBytes; }

int bc_decode_attention_noalloc(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial,
                                int n_slots, int group, int seq_len, int64_t kv_stride, int head_dim, int mode,
                                void* stream) {
    if (n_slots > 0 && valid_group(group) && bc_valid_head_dim(head_dim) && seq_len >= 0 &&
        bc_decode_workspace_bytes(n_slots, group, seq_len, head_dim) > kStaticScratchBytes)
        return BC_ERR_TOO_LARGE;
    if (n_slots <= 0 || !valid_group(group) || !bc_valid_head_dim(head_dim))
        return bc_decode_attention(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim, mode, nullptr,
                                   0, stream);  // argument errors and empty calls, reported as usual
    void* scratch = nullptr;
    int rc = static_scratch_address(&scratch);
    if (rc != BC_OK) return rc;
    // The ticket counters must start at zero.  The array keeps the previous
    // call's contents, and a previous call of another shape may have written
    // partial results over this shape's counters, so they are cleared here.
    const size_t counter_bytes = (size_t)n_slots * (group / heads_per_cta(group)) * sizeof(unsigned);
    cudaError_t e = cudaMemsetAsync(scratch, 0, counter_bytes, (cudaStream_t)stream);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    return bc_decode_attention(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim, mode, scratch,
                               kStaticScratchBytes, stream);
}

}  // extern "C"
