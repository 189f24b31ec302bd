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
// Work decomposition.  A CTA of 4 warps owns one KV slot (batch, kv head), a
// contiguous key range (its split) and GC query heads of that slot's group.
// Tiles of 128 keys stream into a shared-memory ring by 1-D TMA bulk copies
// (cp.async.bulk, no multicast) completing on "full" mbarriers; each warp
// releases a stage through an "empty" mbarrier, so warps never meet at a
// CTA-wide barrier inside the loop.  A warp owns 32 keys of every tile: in
// the score phase each lane scores one key over the whole head, in the value
// phase d/32 lanes share a key (32 dims each).  Each warp keeps one online
// softmax state; warps are merged once per CTA and splits once per slot by
// the last CTA to finish (atomic ticket), so one launch produces the final
// fp16 output.
//
// Scores.  Sign agreement: d - 2*popc(q_sign ^ k_sign) over the head.  The
// INT4 residual dot is exact integer arithmetic: each query element is
// quantised once to 16 bits (q ~= Q16 * qmax/32767) split into hi/lo bytes;
// the plane stores codes offset-binary (u = n + 8), dotted with dp4a (odd
// elements in place as 16u); the offset is removed with a precomputed
// 8*sum(Q16).
//
// Values.  For key weight w: sign part 2*a*b - a with a = w*scale_v, residual
// part c*(u - 8) with c = w*res_scale_v/7 and u = n+8.  Sign bits and nibbles
// are masked in place and used directly as fp32 denormal operands
// (pattern * 2^-149) of packed fma.rn.f32x2 with one coefficient per key;
// each accumulator carries the fixed power-of-two scale of its bit position,
// removed once per CTA together with the constant parts sum_s (a_s + 8 c_s).
#include <cuda.h>

#include <type_traits>
#include <cstring>
#include <mutex>

#include "encode_core.cuh"

namespace bc {

__device__ unsigned int g_bc_device_error = 0;

// Tuning knobs (defaults are the measured best; see the design notes).
#ifndef BC_DEC_STAGES
#define BC_DEC_STAGES 2        // ring stages at head_dim <= 128 (2: 4 CTAs, 16 warps per SM)
#endif
#ifndef BC_DEC_WAVES
#define BC_DEC_WAVES 1         // resident waves of CTAs the split plan aims for
#endif

#ifndef BC_DEC_THREADS
#define BC_DEC_THREADS 128     // threads per CTA (4 warps; each warp owns 32 keys of a tile)
#endif
#ifndef BC_DEC_DL1
#define BC_DEC_DL1 32          // value-phase dims per lane with one head per CTA
#endif
#ifndef BC_DEC_MIN_CTAS_C1
#define BC_DEC_MIN_CTAS_C1 4   // resident CTAs per SM the compensated one-head kernel is held to
#endif
#ifndef BC_DEC_MIN_CTAS_B1
#define BC_DEC_MIN_CTAS_B1 4   // resident CTAs per SM the binary one-head tensor-core kernel is held to (C3 binary: 4 21.4 us, 5 22.9 us)
#endif
#ifndef BC_DEC_BIN_GC
#define BC_DEC_BIN_GC 4        // most query heads per CTA in binary grouped-query caches (binary C4: 4 heads 91 us, 2 heads 106 us)
#endif
#ifndef BC_DEC_GQA_GC
#define BC_DEC_GQA_GC 4        // most query heads per CTA in compensated grouped-query caches at head dims 64 and 128
#endif
#ifndef BC_DEC_KCOMB
#define BC_DEC_KCOMB 8         // split partials each combining thread loads per L2 round trip
#endif
#ifndef BC_DEC_BIN_TPS
#define BC_DEC_BIN_TPS 4       // binary caches, tensor-core path: 128-key tiles per ring stage
#endif
#ifndef BC_DEC_FILL
#define BC_DEC_FILL 1          // plan several waves when one wave leaves CTA slots idle
#endif
#ifndef BC_DEC_MIN_TILES
#define BC_DEC_MIN_TILES 1     // fewest 128-key tiles a split is planned with
#endif
#ifndef BC_DEC_MMA
#define BC_DEC_MMA 1           // value phase on the tensor cores (u8 mma.sync); by-bit planes need it
#endif
constexpr int kDecThreads = BC_DEC_THREADS;
constexpr int kWarps = kDecThreads / 32;
constexpr int kTile = kDecThreads;  // keys per tile: 32 per warp
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLazy = 8.0f;     // rescale only when the running max grows by > 2^8
constexpr int kAccShift = 64;     // accumulators hold value * 2^-64

template <int D, int GC, bool COMP>
struct DecCfg {
    static constexpr int NWD = D / 32;       // sign words (and 16-byte nibble chunks) per key
    // Value phase: each lane accumulates DL dims of a key, 32 with one head per
    // CTA, 16 with several (so GC heads' accumulators fit the register budget).
    static constexpr int DL = (GC == 1) ? BC_DEC_DL1 : 16;
    static constexpr int NP = DL / 2;        // f32x2 accumulator pairs per lane and head part
    static constexpr int QPK = D / DL;       // value-phase lanes per key
    static constexpr int KPW = 32 / QPK;     // value-phase keys in parallel per warp
    static constexpr int NS = (D == 256) ? 2 : BC_DEC_STAGES;  // ring stages
    static constexpr int LAG = 1;            // refill the stage consumed one tile ago
    static constexpr int T = kTile;
    // Tensor-core value phase: the value sums of GC heads are NT column tiles
    // of 8 (two heads x four coefficient bytes each) by NRT row tiles of 16
    // dims.  Compensated caches at head dims 64, 128 (up to four heads per
    // CTA) and 256 (up to two: 64 accumulator registers per head pair),
    // binary ones at head_dim 128.  BM: the binary row map (MmaState).
    static constexpr bool MMA =
        BC_DEC_MMA && ((D == 128 && GC <= 4) || (COMP && ((D == 64 && GC <= 4) || (D == 256 && GC <= 2))));
    static constexpr bool BM = MMA && !COMP;
    static constexpr int NT = (GC + 1) / 2;
    static constexpr int NRT = D / 16;
    // Binary caches on the tensor-core path stage TPS tiles per ring slot (a
    // binary tile is only 4.6 KB at head_dim 128): attention and entropy
    // stream that many per stage, the step and record kernels one.
    static constexpr int TPS = (MMA && !COMP) ? BC_DEC_BIN_TPS : 1;
    static constexpr int KEYS = T * TPS;     // keys a stage can hold
    static constexpr int SIGN_B = KEYS * D / 8;
    static constexpr int NIB_B = COMP ? T * D / 2 : 0;
    static constexpr int SC_B = KEYS * 2;
    static constexpr int OFF_KSIGN = 0;
    static constexpr int OFF_KBS = OFF_KSIGN + SIGN_B;
    static constexpr int OFF_KNIB = OFF_KBS + SC_B;
    static constexpr int OFF_KRS = OFF_KNIB + NIB_B;
    static constexpr int OFF_VSIGN = OFF_KRS + (COMP ? SC_B : 0);
    static constexpr int OFF_VBS = OFF_VSIGN + SIGN_B;
    static constexpr int OFF_VNIB = OFF_VBS + SC_B;
    static constexpr int OFF_VRS = OFF_VNIB + NIB_B;
    static constexpr int STAGE_B = OFF_VRS + (COMP ? SC_B : 0);
    static constexpr int RING_B = NS * STAGE_B;
    static constexpr int MERGE_B = kWarps * GC * (D + 2) * 4;  // reuses the ring after the main loop
    // tensor-core value phase: the warps' accumulators are dumped after the
    // merge records ([warp][lane][NT * NRT * 4 + 1] ints) for the final read-out
    static constexpr int DUMP_STRIDE = NT * NRT * 4 + 1;
    static constexpr int DUMP_OFF = (MERGE_B + 127) & ~127;
    static constexpr int DUMP_B = kWarps * 32 * DUMP_STRIDE * 4;
    // the ring, reused after the main loop by the merge records and the dump
    static constexpr int AFTER_B = MMA ? DUMP_OFF + DUMP_B : MERGE_B;
    static constexpr int BODY_B = RING_B > AFTER_B ? RING_B : AFTER_B;
    static constexpr int QSIGN_OFF = BODY_B;                    // uint32 [GC][8]
    static constexpr int QCONST_OFF = QSIGN_OFF + GC * 8 * 4;   // [GC][4]: bco, rco, off8, eco
    // the residual score's query operand: dp4a packs, uint32 [GC][D/8][4]
    // (the record kernel), and on the tensor-core path the A matrix of the
    // score MMA, [D/32 chunks][2][16 rows][16 B]
    static constexpr int QPK_OFF = QCONST_OFF + GC * 4 * 4;
    static constexpr int QPK_DP4A_B = GC * (D / 8) * 16;
    static constexpr int QPK_B = (MMA && D * 16 > QPK_DP4A_B) ? D * 16 : QPK_DP4A_B;
    static constexpr int FULL_OFF = QPK_OFF + QPK_B;            // mbarriers
    static constexpr int EMPTY_OFF = FULL_OFF + NS * 8;         // mbarriers: all warps done with a stage
    static constexpr int FLAG_OFF = EMPTY_OFF + NS * 8;         // abort flag
    // Fused decode step: the appended K and V rows, staged once per CTA in
    // plane format (sign words, 16-byte nibble chunks in natural order, scales).
    static constexpr int NEWSIGN_B = (D / 8 + 15) & ~15;
    static constexpr int NEWROW_B = NEWSIGN_B + D / 2 + 16;
    static constexpr int NEW_OFF = FLAG_OFF + 16;               // [2][NEWROW_B]: K row, V row
    static constexpr int NEWRAW_OFF = NEW_OFF + 2 * NEWROW_B;   // fp16 [2][D]: the new K, V rows as given
    // Scratch used either before the main loop (query preparation: q as
    // float [GC][D], then Q16 int [GC][D]) or inside it (tensor-core path,
    // per warp: the fixed-point key coefficients as bytes, [part: sign,
    // code][8 NT rows: head * 4 + byte][48], and the residual score dots of
    // the warp's 32 keys, int [GC][40]), never both at once.
    static constexpr int SCR_OFF = NEWRAW_OFF + 4 * D;
    static constexpr int QF_OFF = SCR_OFF;
    static constexpr int Q16_OFF = QF_OFF + GC * D * 4;
    static constexpr int WB_ROW = 48;                           // padded: the fragment loads hit distinct banks
    static constexpr int WB_PART = 8 * NT * WB_ROW;
    static constexpr int WB_WARP = 2 * WB_PART;
    static constexpr int DOT_WARP = GC * 40 * 4;
    static constexpr int WB_OFF = SCR_OFF;
    static constexpr int DOT_OFF = WB_OFF + (MMA ? kWarps * WB_WARP : 0);
    static constexpr int LOOP_SCR_B = MMA ? kWarps * (WB_WARP + DOT_WARP) : 0;
    static constexpr int SCR_B = LOOP_SCR_B > 2 * GC * D * 4 ? LOOP_SCR_B : 2 * GC * D * 4;
    static constexpr int SMEM_B = SCR_OFF + SCR_B + 128;       // + slack to align the base to 128 B
    static_assert(!MMA || DUMP_OFF + DUMP_B <= BODY_B, "accumulator dump exceeds the ring");
    // Resident CTAs per SM that shared memory allows at head_dim <= 128 with one
    // head per CTA; the register budget is held to it.
    // (head_dim 64, one head: five, whose registers then match the five
    // CTAs that shared memory allows)
    // (head_dim 256, compensated: two, which shared memory allows anyway, so
    // the kernel may use up to 255 registers: C5 d=256 466 -> 455 us against
    // the compiler's own choice of 128; binary: no bound, the compiler's choice)
    static constexpr int MIN_CTAS =
        (D > 128) ? (COMP ? 2 : 0)
                  : ((GC == 1 && !COMP) ? (D == 128 ? BC_DEC_MIN_CTAS_B1 : 5)
                                        : (GC == 1 ? (D == 64 ? 5 : BC_DEC_MIN_CTAS_C1) : 4)) * 128 / kDecThreads;
};

struct DecodeArgs {
    const __half* q;    // [n_slots * group][d]
    bc_kv_planes K, V;  // planes, or record bases in .sign (bin) / .nib (res) for the record kernel
    __half* out;        // [n_slots * group][d] or null
    float* partial;     // [n_slots * group][d + 2] or null
    float* ws_part;     // [n_slots * group][n_splits][d + 4]: m, l, 2 pad, o[d] (o 16-byte aligned)
    unsigned* ws_cnt;   // [n_slots * n_hgroups]
    int n_slots, group, seq_len, n_splits, keys_per_split, n_hgroups;
    int64_t kv_stride;
    int head_dim;
    // fused decode step only: one new K and V row per slot, written at plane
    // position append_pos of every slot before that position is attended
    const __half* new_k;
    const __half* new_v;
    int append_pos, append_res;
    int host_in;        // fused step: bit 0 q, bit 1 new_k / new_v are in pinned host memory
    // paged caches (pages != null): logical position s of slot j lives in plane
    // row pages[j * max_pages + s / page_size] * page_size + s % page_size
    const int* pages;
    int max_pages, page_size, n_pages;
    // entropy variant: per query head H of the softmax over the binary scores
    // without 1/sqrt(d) (reference adaptive_precision.cu:13-130)
    float* entropy;  // [n_slots * group]
    float* ws_ent;   // [n_slots * group][n_splits][3] split partials (m, z, w)
    // compact adaptive caches (VAR 3): positions [0, n_keep) of a slot carry
    // residuals (residual planes at row stride res_stride); the binary-only
    // rest sits at sign/scale rows [b0, b0 + seq_len - n_keep).  Splits
    // [0, nc) cover the first segment with keys_per_split keys each, the
    // remaining splits the second with kps_bin keys each.
    int n_keep, nc, kps_bin, b0;
    int64_t res_stride;
    // sequence split over peer memory (xw > 0): the final (m, l, o) of every
    // head goes straight into every rank's exchange buffer as 64-bit words
    // (value, epoch), and each rank merges the xw partials itself once every
    // word it needs carries the call's epoch
    unsigned long long* xparts[8];  // rank j's buffer as mapped here: [2 parities][xw][n_heads][d+2]
    int xw, xrank;
    unsigned xepoch;
    unsigned xspin;  // polls of one exchange word before the CTA gives up
};

// Plane row of logical position `pos` of `slot`, or -1 for a page id outside
// the pool (the caller reports BC_DEVERR_PAGE instead of touching memory).
__device__ __forceinline__ int64_t plane_row(const DecodeArgs& a, int slot, int pos) {
    if (!a.pages) return (int64_t)slot * a.kv_stride + pos;
    const int pg = __ldg(a.pages + (int64_t)slot * a.max_pages + pos / a.page_size);
    return (pg >= 0 && pg < a.n_pages) ? (int64_t)pg * a.page_size + pos % a.page_size : -1;
}

// Per-lane query state for GC heads.  The score phase handles whole keys, so
// every lane holds the full query: sign words and, for the residual dot, q
// quantised to 16 bits split into hi (signed) / lo (unsigned) bytes, packed
// per nibble word as [even hi, even lo, odd hi, odd lo].
template <int D, int GC>
struct QState {
    uint32_t sign[GC][D / 32];
    const uint4* pk;  // shared memory, [GC][D/8]
    float bco[GC], rco[GC];
    int off8[GC];
    float eco[GC];  // entropy variant: the query's tree-order mean |q| (adaptive_precision.cu:46-59)
};

// Value accumulators.  Pair p holds dims (p, p + NP) of the lane's DL-dim
// chunk.  Sign part: sum of 2a*b (a = w*scale_v) scaled by 2^(p-64), because
// sign bit p enters as the denormal 2^(p-149) and the coefficient is the
// same 2a*2^85 for every p.  Residual part: sum of c*u (c = w*res_scale_v/7,
// u = code + 8) scaled by 2^(4(p%4) - 64), the nibble's in-register position
// (nibbles 4-7 of a word are taken from its upper half, which keeps every
// masked field below bit 23, the linear denormal range).  Keeping the two
// parts apart lets every FFMA2 of a key share one coefficient; the fixed
// scales are removed once per CTA.
template <int GC, int NP>
struct SoftState {
    float m[GC];         // running max (log2 units), uniform across the warp
    float l[GC], t[GC];  // per lane: sum of weights and sum of (a + 8c) of the lane's own keys
    f2 acc_s[GC][NP];    // sign part
    f2 acc_n[GC][NP];    // residual part
    float em[GC], ez[GC], ew[GC];  // entropy variant, per lane: max, sum e^(s-max), sum e^(s-max) s
};

__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 127) & ~uintptr_t(127));
}

// ---------------------------------------------------------------------------
// Query preparation (once per CTA).  scale_q is summed sequentially over the
// head as in compensated_attention.cu:65-67.  The residual dot uses q
// quantised against the head's max |q|: q_i ~= Q16_i * qmax / 32767.
// ---------------------------------------------------------------------------
// 16-byte asynchronous global->shared copies (cp.async, no register staging).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Start the copy of the CTA's query rows (fp16) into the Q16 area before the
// ring's first bulk copies are issued, so the few hundred bytes of q are not
// queued behind them.  Returns false (nothing issued) when the rows are not
// 16-byte aligned; prepare_query then loads them directly.
template <int D, int GC, typename Cfg>
__device__ __forceinline__ bool prefetch_query(const DecodeArgs& a, int slot, int hg, uint8_t* smem) {
    const __half* src = a.q + ((int64_t)slot * a.group + (int64_t)hg * GC) * D;
    if ((reinterpret_cast<uintptr_t>(src) & 15) != 0) return false;
    for (int c = threadIdx.x; c < GC * D / 8; c += kDecThreads) cp_async16(smem + Cfg::Q16_OFF + 16 * c, src + 8 * c);
    asm volatile("cp.async.commit_group;" ::: "memory");
    return true;
}

// QMMA: the residual score runs on the tensor cores (by-bit planes): q is
// quantised to |Q16| <= 32639 and split into balanced digits Q16 = 256 hi + lo
// with hi, lo in [-128, 127] (s8 operands); the A matrix of the score MMA,
// [chunk c][half h][row][16 bytes], holds at byte k of row g (head g's hi
// digit) / row 8 + g (its lo digit) the digit of dim nib_dim(D, c, k, h), the
// dim of byte k of nibble chunk c (low nibble for h = 0, high for h = 1).
// Otherwise q is quantised to |Q16| <= 32767 and packed for dp4a.
template <int D, int GC, bool COMP, typename Cfg, bool QMMA = false>
__device__ __forceinline__ void prepare_query(const DecodeArgs& a, int slot, int hg, uint8_t* smem,
                                              QState<D, GC>& qs, bool staged = false) {
    constexpr float kQMax = QMMA ? 32639.0f : 32767.0f;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* qf = reinterpret_cast<float*>(smem + Cfg::QF_OFF);
    int* q16 = reinterpret_cast<int*>(smem + Cfg::Q16_OFF);
    uint32_t* qsign = reinterpret_cast<uint32_t*>(smem + Cfg::QSIGN_OFF);
    float* qc = reinterpret_cast<float*>(smem + Cfg::QCONST_OFF);
    const int64_t qbase = ((int64_t)slot * a.group + (int64_t)hg * GC) * D;
    if (staged) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        const __half* st = reinterpret_cast<const __half*>(smem + Cfg::Q16_OFF);
        for (int i = tid; i < GC * D; i += kDecThreads) qf[i] = __half2float(st[i]);
    } else {
        for (int i = tid; i < GC * D; i += kDecThreads) qf[i] = __half2float(a.q[qbase + i]);
    }
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
        const float qscale = mx > 0.0f ? kQMax / mx : 0.0f;
        int sum16 = 0;
        for (int k = 0; k < D / 32; ++k) {
            const int v = __float2int_rn(qf[g * D + 32 * k + lane] * qscale);
            q16[g * D + 32 * k + lane] = v;
            sum16 += v;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum16 += __shfl_xor_sync(0xffffffffu, sum16, off);
        // scale_q: a sequential sum in element order; the elements come from
        // the lanes by shuffle so their loads do not sit on the add chain
        float sq = 0.0f;
#pragma unroll 1
        for (int k = 0; k < D / 32; ++k) {
            const float v = fabsf(qf[g * D + 32 * k + lane]);
#pragma unroll
            for (int j = 0; j < 32; ++j) sq += __shfl_sync(0xffffffffu, v, j);
        }
        {
            // entropy scale: the reference block's strided sums and stride-halving tree
            float x[D / 32];
#pragma unroll
            for (int k = 0; k < D / 32; ++k) x[k] = qf[g * D + 32 * k + lane];
            const float te = tree_abs_sum<D / 32>(x) / (float)D;
            if (lane == 0) qc[g * 4 + 3] = te;
        }
        if (lane == 0) {
            sq /= (float)D;
            qc[g * 4 + 0] = sq * inv_sqrt_d * kLog2e;
            qc[g * 4 + 1] = (mx / kQMax) * (1.0f / 7.0f) * inv_sqrt_d * kLog2e;
            reinterpret_cast<int*>(qc)[g * 4 + 2] = 8 * sum16;
        }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GC; ++g) {
#pragma unroll
        for (int k = 0; k < D / 32; ++k) qs.sign[g][k] = qsign[g * 8 + k];
        qs.bco[g] = qc[g * 4 + 0];
        qs.rco[g] = qc[g * 4 + 1];
        qs.off8[g] = reinterpret_cast<const int*>(qc)[g * 4 + 2];
        qs.eco[g] = qc[g * 4 + 3];
        qs.pk = reinterpret_cast<const uint4*>(smem + Cfg::QPK_OFF);
        if (COMP && !QMMA) {
            uint4* dst = reinterpret_cast<uint4*>(smem + Cfg::QPK_OFF);
            for (int w = threadIdx.x; w < D / 8; w += kDecThreads) {
                uint32_t eh = 0, el = 0, oh = 0, ol = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int ve = q16[g * D + 8 * w + 2 * b], vo = q16[g * D + 8 * w + 2 * b + 1];
                    eh |= ((uint32_t)(ve >> 8) & 0xFFu) << (8 * b);
                    el |= ((uint32_t)ve & 0xFFu) << (8 * b);
                    oh |= ((uint32_t)(vo >> 8) & 0xFFu) << (8 * b);
                    ol |= ((uint32_t)vo & 0xFFu) << (8 * b);
                }
                dst[g * (D / 8) + w] = make_uint4(eh, el, oh, ol);
            }
        }
    }
    if constexpr (QMMA && COMP) {
        static_assert(nib_by_bit(D) && GC <= 8, "score MMA: by-bit planes, at most 8 heads");
        uint32_t* qa = reinterpret_cast<uint32_t*>(smem + Cfg::QPK_OFF);
        for (int w = threadIdx.x; w < D * 4; w += kDecThreads) {  // word w: chunk, half, row, bytes 4k4..4k4+3
            const int k4 = w & 3, row = (w >> 2) & 15, h = (w >> 6) & 1, c = w >> 7;
            const int g = row & 7;
            uint32_t word = 0;
            if (g < GC) {
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int v = q16[g * D + nib_dim(D, c, 4 * k4 + b, h)];
                    const int lo = ((v + 128) & 255) - 128, hi = (v - lo) >> 8;
                    word |= ((uint32_t)(row < 8 ? hi : lo) & 0xFFu) << (8 * b);
                }
            }
            qa[w] = word;
        }
    }
    __syncthreads();
}

template <int GC, int NP>
__device__ __forceinline__ void init_soft(SoftState<GC, NP>& st) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        st.m[g] = -INFINITY;
        st.l[g] = 0.0f;
        st.t[g] = 0.0f;
        st.em[g] = -INFINITY;
        st.ez[g] = 0.0f;
        st.ew[g] = 0.0f;
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            st.acc_s[g][p] = f2{0.0f, 0.0f};
            st.acc_n[g][p] = f2{0.0f, 0.0f};
        }
    }
}

// State of the tensor-core value phase.  The value sums live in integer MMA
// accumulators: acc[n][t] is the m16n8 tile t (rows = dims, see
// consume_warp_tile_mma) of column tile n (columns = head 2n + col / 4, byte
// col % 4 of the key coefficient).  The sign bits and the INT4 codes of a dim
// share its accumulator row: the sign bit enters with the coefficient 2 e
// bscale, the code with e rscale / 7, both as 32-bit fixed-point numbers split
// into four byte columns, where e = 2^(s - U[g]) is the key's softmax weight
// in units of 2^U[g] (absolute, log2).  U is the softmax's running reference
// point as well: the weight sum l and the constant term t are kept in the
// same units, so there is no separate running max.  U moves only when a
// coefficient would reach 2^31 units; the accumulators are then shifted down
// exactly and l, t scaled by the same power of two.
constexpr int kUUnset = -0x40000000;

// NRT: row tiles (head_dim / 16).
template <int GC, int NRT = 8>
struct MmaState {
    static constexpr int NT = (GC + 1) / 2;
    float Uf[GC];  // U as a float, -inf while unset
    float l[GC], t[GC];
    int acc[NT][NRT][4];
    int U[GC];
    float em[GC], ez[GC], ew[GC];
};

template <int GC, int NRT>
__device__ __forceinline__ void init_soft(MmaState<GC, NRT>& st) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        st.Uf[g] = -INFINITY;
        st.l[g] = 0.0f;
        st.t[g] = 0.0f;
        st.U[g] = kUUnset;
        st.em[g] = -INFINITY;
        st.ez[g] = 0.0f;
        st.ew[g] = 0.0f;
    }
#pragma unroll
    for (int n = 0; n < MmaState<GC, NRT>::NT; ++n)
#pragma unroll
        for (int t = 0; t < NRT; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) st.acc[n][t][i] = 0;
}

// ---------------------------------------------------------------------------
// One warp consumes its 32 keys of a tile held in shared memory (canonical
// layout: sign rows, bscale, interleaved offset-binary nibbles, rscale; K then V).
//  1. score phase: lane `lane` scores key `kw + lane` for the GC heads;
//  2. lazy rescale of the warp's running max (vote, then a warp max only when
//     some score exceeds the max by more than 2^8);
//  3. value phase: d/32 lanes per key accumulate 32 dims each (consecutive
//     lanes take consecutive keys, so the interleaved nibble reads are
//     bank-conflict free), receiving the key's weight coefficients from its
//     score lane by shuffle.
// Nibbles are stored offset-binary (u = code + 8), so no XOR is needed here.
// ---------------------------------------------------------------------------
// Score phase of one lane: key kk of the stage for the GC heads (scores in
// log2 units, -inf for keys past the tile's end); the entropy variant also
// folds the binary score into the lane's online entropy state.
template <int D, int GC, bool COMP, typename Cfg, bool ENT, typename St>
__device__ __forceinline__ void score_keys(const QState<D, GC>& qs, St& st, const uint8_t* sb, int kk, bool valid,
                                           float (&s2)[GC]) {
    constexpr int NWD = Cfg::NWD;
    // ---- score phase -------------------------------------------------------
    uint32_t ks[NWD];
    {
        const uint32_t* row = reinterpret_cast<const uint32_t*>(sb + Cfg::OFF_KSIGN) + kk * NWD;
        if constexpr (NWD % 4 == 0) {
#pragma unroll
            for (int c = 0; c < NWD / 4; ++c) {
                const uint4 v = reinterpret_cast<const uint4*>(row)[c];
                ks[4 * c] = v.x; ks[4 * c + 1] = v.y; ks[4 * c + 2] = v.z; ks[4 * c + 3] = v.w;
            }
        } else if constexpr (NWD == 2) {
            const uint2 v = *reinterpret_cast<const uint2*>(row);
            ks[0] = v.x; ks[1] = v.y;
        } else {
            ks[0] = row[0];
        }
    }
    const float kbs = __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_KBS)[kk]);
    int dot[GC];
    float krs = 0.0f;
    if (COMP) {
        krs = __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_KRS)[kk]);
        int eh[GC], el[GC], oh[GC], ol[GC];
#pragma unroll
        for (int g = 0; g < GC; ++g) eh[g] = el[g] = oh[g] = ol[g] = 0;
#pragma unroll
        for (int c = 0; c < NWD; ++c) {
            const uint4 ch = *reinterpret_cast<const uint4*>(sb + Cfg::OFF_KNIB + nib_chunk_offset(kk, c, D));
            const uint32_t wds[4] = {ch.x, ch.y, ch.z, ch.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const uint32_t ue = wds[w] & 0x0F0F0F0Fu;    // even elements, u
                const uint32_t uo16 = wds[w] & 0xF0F0F0F0u;  // odd elements, 16u
#pragma unroll
                for (int g = 0; g < GC; ++g) {
                    const uint4 pv = qs.pk[g * (D / 8) + 4 * c + w];
                    const uint32_t pk[4] = {pv.x, pv.y, pv.z, pv.w};
                    eh[g] = dp4a_us(ue, pk[0], eh[g]);
                    el[g] = dp4a_uu(ue, pk[1], el[g]);
                    oh[g] = dp4a_us(uo16, pk[2], oh[g]);
                    ol[g] = dp4a_uu(uo16, pk[3], ol[g]);
                }
            }
        }
#pragma unroll
        for (int g = 0; g < GC; ++g) dot[g] = eh[g] * 256 + el[g] + ((oh[g] * 256 + ol[g]) >> 4);
    }
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        int pop = 0;
#pragma unroll
        for (int k = 0; k < NWD; ++k) pop += __popc(qs.sign[g][k] ^ ks[k]);
        float s = qs.bco[g] * kbs * (float)(D - 2 * pop);
        if (COMP) s = fmaf(qs.rco[g] * krs, (float)(dot[g] - qs.off8[g]), s);
        s2[g] = valid ? s : -INFINITY;
        if constexpr (ENT) {
            // xnor_dot without 1/sqrt(d), online per lane (adaptive_precision.cu:69-102)
            if (valid) {
                const float sc = qs.eco[g] * kbs * (float)(D - 2 * pop);
                if (sc > st.em[g]) {
                    const float f = (st.em[g] == -INFINITY) ? 0.0f : __expf(st.em[g] - sc);
                    st.ez[g] = st.ez[g] * f + 1.0f;
                    st.ew[g] = st.ew[g] * f + sc;
                    st.em[g] = sc;
                } else {
                    const float e = __expf(sc - st.em[g]);
                    st.ez[g] += e;
                    st.ew[g] += e * sc;
                }
            }
        }
    }
}

template <int D, int GC, bool COMP, typename Cfg, bool ENT = false>
__device__ __forceinline__ void consume_warp_tile(const QState<D, GC>& qs, SoftState<GC, Cfg::NP>& st,
                                                  const uint8_t* sb, int kw, int nk) {
    constexpr int NWD = Cfg::NWD, QPK = Cfg::QPK, KPW = Cfg::KPW, NP = Cfg::NP;
    const int lane = threadIdx.x & 31;
    const int kk = kw + lane;
    const bool valid = kk < nk;
    float s2[GC];
    score_keys<D, GC, COMP, Cfg, ENT>(qs, st, sb, kk, valid, s2);
    // ---- lazy rescale, weights -------------------------------------------------
    const float vbs = valid ? __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_VBS)[kk]) : 0.0f;
    const float vrs = (COMP && valid) ? __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_VRS)[kk]) : 0.0f;
    float A0[GC], C0[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        if (__any_sync(0xffffffffu, s2[g] > st.m[g] + kLazy)) {  // warp-uniform, rare after the first tile
            float M = s2[g];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            const float alpha = fast_exp2(st.m[g] - M);
            st.m[g] = M;
            st.l[g] *= alpha;
            st.t[g] *= alpha;
            const f2 al = {alpha, alpha};
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                fmul2(st.acc_s[g][p], al);
                if constexpr (COMP) fmul2(st.acc_n[g][p], al);
            }
        }
        const float wt = valid ? fast_exp2(s2[g] - st.m[g]) : 0.0f;
        st.l[g] += wt;
        const float av = wt * vbs;
        A0[g] = 2.0f * av * exp2i(149 - kAccShift);
        if (COMP) {
            const float cv = wt * vrs * (1.0f / 7.0f);
            C0[g] = cv * exp2i(149 - kAccShift);
            st.t[g] += av + 8.0f * cv;
        } else {
            C0[g] = 0.0f;
            st.t[g] += av;
        }
    }
    // ---- value phase -----------------------------------------------------------
    const int grp = lane % KPW, qt = lane / KPW;
    if constexpr (Cfg::DL == 32) {
#pragma unroll
        for (int r = 0; r < QPK; ++r) {
            const int src = grp + r * KPW;
            const int kv = kw + src;
            const uint32_t vs = reinterpret_cast<const uint32_t*>(sb + Cfg::OFF_VSIGN)[kv * NWD + qt];
            const uint32_t vs_hi = vs >> 16;
            uint32_t nw[4] = {0, 0, 0, 0}, nh[4] = {0, 0, 0, 0};
            if (COMP) {
                const uint4 vn = *reinterpret_cast<const uint4*>(sb + Cfg::OFF_VNIB + nib_chunk_offset(kv, qt, D));
                nw[0] = vn.x; nw[1] = vn.y; nw[2] = vn.z; nw[3] = vn.w;
#pragma unroll
                for (int k = 0; k < 4; ++k) nh[k] = nw[k] >> 16;
            }
#pragma unroll
            for (int g = 0; g < GC; ++g) {
                const float a0 = __shfl_sync(0xffffffffu, A0[g], src);
                const float c0 = COMP ? __shfl_sync(0xffffffffu, C0[g], src) : 0.0f;
                const f2 a2 = {a0, a0}, c2 = {c0, c0};
#pragma unroll
                for (int p = 0; p < 16; ++p) {
                    // sign bits of dims p and p+16, each the exact denormal 2^(p-149)
                    const f2 y = {bits_f(vs & (1u << p)), bits_f(vs_hi & (1u << p))};
                    ffma2(st.acc_s[g][p], a2, y);
                    if (COMP) {
                        // codes of dims p (word p/8) and p+16 (word 2 + p/8), nibble p%8:
                        // nibbles 0-3 from the word, 4-7 from its upper half
                        const int t = p & 7, kw0 = p >> 3;
                        const uint32_t srca = (t < 4) ? nw[kw0] : nh[kw0];
                        const uint32_t srcb = (t < 4) ? nw[2 + kw0] : nh[2 + kw0];
                        const int sh = 4 * (t & 3);
                        const f2 x = {bits_f(srca & (0xFu << sh)), bits_f(srcb & (0xFu << sh))};
                        ffma2(st.acc_n[g][p], c2, x);
                    }
                }
            }
        }
    } else {
        // 16-dim lanes: lane (grp, qt) takes half qt%2 of chunk qt/2.  Within
        // each 8-key block the chunks alternate between the block's key groups
        // round by round, so one round's 8-byte nibble loads cover all banks.
        constexpr int G = KPW < 8 ? 8 / KPW : 1;  // key groups per 8-key block
        const int c = qt >> 1, h = qt & 1;
#pragma unroll
        for (int r = 0; r < QPK; ++r) {
            const int src = (G > 1) ? 8 * (r / G) + KPW * ((r + c) % G) + grp : grp + r * KPW;
            const int kv = kw + src;
            const uint32_t vs = reinterpret_cast<const uint32_t*>(sb + Cfg::OFF_VSIGN)[kv * NWD + c] >> (16 * h);
            const uint32_t vs_hi = vs >> 8;
            uint32_t n0 = 0, n1 = 0, nh0 = 0, nh1 = 0;
            if (COMP) {
                const uint2 vn = *reinterpret_cast<const uint2*>(sb + Cfg::OFF_VNIB + nib_chunk_offset(kv, c, D) + 8 * h);
                n0 = vn.x;
                n1 = vn.y;
                nh0 = n0 >> 16;
                nh1 = n1 >> 16;
            }
#pragma unroll
            for (int g = 0; g < GC; ++g) {
                const float a0 = __shfl_sync(0xffffffffu, A0[g], src);
                const float c0 = COMP ? __shfl_sync(0xffffffffu, C0[g], src) : 0.0f;
                const f2 a2 = {a0, a0}, c2 = {c0, c0};
#pragma unroll
                for (int p = 0; p < 8; ++p) {
                    // sign bits of dims p and p+8; codes of dims p (word 0) and p+8
                    // (word 1), nibble p: nibbles 4-7 from the words' upper halves, so
                    // every masked field stays in the fp32 denormal range (bits < 23)
                    const f2 y = {bits_f(vs & (1u << p)), bits_f(vs_hi & (1u << p))};
                    ffma2(st.acc_s[g][p], a2, y);
                    if (COMP) {
                        const int sh = 4 * (p & 3);
                        const f2 x = {bits_f((p < 4 ? n0 : nh0) & (0xFu << sh)), bits_f((p < 4 ? n1 : nh1) & (0xFu << sh))};
                        ffma2(st.acc_n[g][p], c2, x);
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Tensor-core path (written out here for head_dim 128; 256 and 64 below).
//
// Score: the XNOR popcount stays on SIMT, one lane per key.  The INT4
// residual dot sum_d u_d Q16_d of the warp's 32 keys and all GC heads is one
// set of d / 8 mma.sync m16n8k32 s8 x u8 -> s32 (residual_dots_mma): A = the
// query's balanced hi/lo digits (rows), B = the offset-binary codes (keys).
//
// Values: per warp and tile, D[dims x (head, byte)] += A[dims x 32 keys] .
// W[32 keys x (head, byte)] with mma.sync m16n8k32 u8 x u8 -> s32; lane =
// 4 g8 + q, MMA k index = the warp's key.  ldmatrix .m16n16 .trans .b8 on 16
// keys x 16 bytes hands lane (g8, q) byte g8 (and g8 + 8) of keys 4q .. 4q + 3,
// so one shift and mask per fragment remain.  Row tile t = 2c + h has
//   row g8     = dim 64 h + 8 g8 + c      (one unit per unit of the operand)
//   row g8 + 8 = dim 64 h + 8 g8 + c + 4  (16 units per unit)
// for both parts: sign bit c (row g8 + 8: bit c + 4) of sign byte g8 + 8h,
// shifted down by c and masked with 0x01 (0x10) per byte; and the low (high)
// nibble of byte g8 + 8h of nibble chunk c, which in the by-bit nibble order
// holds exactly those two dims.  So the sign bits and the codes of a dim
// accumulate in the same row, with the sign coefficient 2 e bscale and the
// code coefficient e rscale / 7 as their B operands (e = 2^(s - U), the key's
// weight in the fixed-point unit: see MmaState).  Each lane writes its
// key's fixed-point coefficient bytes to the warp's scratch
// ([part][head * 4 + byte][key]) and reads its B fragments (column g8 of
// column tile n: head 2n + g8 / 4, byte g8 % 4; keys 4q.., 4q + 16..) as two
// 32-bit words.
//
// head_dim 256: the same for each 16-byte window w of the 32-byte sign row:
// row tile 8w + 2c + h holds dims 128w + 64h + 8g8 + c (+ 4), sign byte
// 16w + 8h + g8 and nibble chunk 4w + c.
// head_dim 64: the sign row is 8 bytes, so one ldmatrix .m16n16 .x1 .trans on
// the warp's 256 sign bytes, read as 16 rows of two keys, hands lane (g8, q)
// byte g8 of keys 8q + 2i (first register) and 8q + 2i + 1 (second), i < 4.
// Row tile t (< 4) holds dims 8g8 + t (row g8) and 8g8 + t + 4 (row g8 + 8):
// sign bits t and t + 4 of byte g8, and the two nibbles of byte 8 (t % 2) + g8
// of chunk t / 2 (by-bit order at 64).  The sign fragments take the keys in
// the order above, so the sign coefficients are written to the scratch at the
// matching MMA k index (sign_k), the code coefficients in key order.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 16x16 byte matrix, transposed: lanes 0-15 give its rows; lane (g8, q)
// receives bytes 4q .. 4q + 3 of columns g8 (r0) and g8 + 8 (r1).
__device__ __forceinline__ void ldsm_x1_trans_b8(const uint8_t* row, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m16n16.x1.trans.shared.b8 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(smem_u32(row)));
}

// Two 16x16 byte matrices, transposed: lanes 0-15 give the rows of the first,
// lanes 16-31 those of the second; r0, r1 come from the first.
__device__ __forceinline__ void ldsm_x2_trans_b8(const uint8_t* row, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                 uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(row)));
}

// Four 8x8 b16 matrices (rows of 16 bytes; lanes 8i .. 8i + 7 give the rows of
// matrix i): lane (g8, q) receives bytes 4q .. 4q + 3 of row g8 of each.
__device__ __forceinline__ void ldsm_x4(const uint8_t* row, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(row)));
}

// Where the tensor-core path finds the CTA's query state (shared memory):
// sign words [GC][8], constants [GC][4] (bco, rco, off8 as int, eco) and the A
// matrix of the score MMA (see prepare_query).
struct QSmem {
    const uint32_t* sign;
    const float* c;
    const uint8_t* qa;
};

constexpr int kDotRow = 40;  // ints per head row of a warp's dot buffer (padded: conflict-free stores)

// Residual dots of the warp's keys kw .. kw + 31 for GC heads:
// dotb[g * kDotRow + key] = sum_d u_d Q16_d (u = code + 8).  B fragments:
// chunk c of an 8-key block is 8 consecutive 16-byte rows; lane (g8, q) gets
// bytes 4q .. 4q + 3 of key g8, whose low nibbles are the k = 4q.. elements
// and whose high nibbles, shifted down, the k = 16 + 4q.. elements of the
// chunk's A matrix.  D rows g / 8 + g are head g's hi / lo digit, columns
// the keys, so dot = 256 D[g] + D[8 + g] stays in one lane.  One x4 load
// takes four chunks of a block (head_dim >= 128) or both chunks of two
// blocks (head_dim 64).
template <int D, int GC>
__device__ __forceinline__ void residual_dots_mma(const uint8_t* knib, int kw, const uint8_t* qa, int* dotb) {
    constexpr int NCH = D / 32, CG = NCH < 4 ? NCH : 4;
    const int lane = threadIdx.x & 31, g8 = lane >> 2, q = lane & 3, mi = lane >> 3;
    const uint8_t* kb = knib + (kw >> 3) * (4 * D) + 16 * (lane & 7);
    int acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0;
#pragma unroll
    for (int c0 = 0; c0 < NCH; c0 += CG) {
        uint32_t a[CG][4];
#pragma unroll
        for (int c = 0; c < CG; ++c)
            ldsm_x4(qa + ((2 * (c0 + c) + (lane >> 4)) * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * 16, a[c][0],
                    a[c][1], a[c][2], a[c][3]);
        if constexpr (NCH >= 4) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t nb[4];
                ldsm_x4(kb + j * (4 * D) + 128 * (c0 + mi), nb[0], nb[1], nb[2], nb[3]);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    mma_s8u8(acc[j], a[c][0], a[c][1], a[c][2], a[c][3], nb[c] & 0x0F0F0F0Fu, (nb[c] >> 4) & 0x0F0F0F0Fu);
            }
        } else {  // head_dim 64: matrix mi = block 2jj + mi / 2, chunk mi % 2
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                uint32_t nb[4];
                ldsm_x4(kb + (2 * jj + (mi >> 1)) * (4 * D) + 128 * (mi & 1), nb[0], nb[1], nb[2], nb[3]);
#pragma unroll
                for (int m = 0; m < 4; ++m)
                    mma_s8u8(acc[2 * jj + (m >> 1)], a[m & 1][0], a[m & 1][1], a[m & 1][2], a[m & 1][3],
                             nb[m] & 0x0F0F0F0Fu, (nb[m] >> 4) & 0x0F0F0F0Fu);
            }
        }
    }
    if (g8 < GC)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<int2*>(dotb + g8 * kDotRow + 8 * j + 2 * q) =
                make_int2(acc[j][0] * 256 + acc[j][2], acc[j][1] * 256 + acc[j][3]);
}

// Divide head g's accumulators by 2^delta (delta >= 1), exactly up to the
// dropped low bits: each (row, tile) value is rebuilt from its four byte
// columns (lanes with q = 2 (g % 2), 2 (g % 2) + 1 of column tile g / 2),
// shifted, and split back into byte columns.
template <int GC, int NRT>
__device__ __forceinline__ void mma_shift_down(MmaState<GC, NRT>& st, int g, int delta) {
    const int q = threadIdx.x & 3;
    const bool mine = (q >> 1) == (g & 1), upper = q & 1;
    const int n = g >> 1;
#pragma unroll
    for (int t = 0; t < NRT; ++t)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint64_t v = (uint64_t)(uint32_t)st.acc[n][t][2 * r] + ((uint64_t)(uint32_t)st.acc[n][t][2 * r + 1] << 8);
            const uint64_t vn = __shfl_xor_sync(0xffffffffu, v, 1);
            const uint64_t lo = upper ? vn : v, hi = upper ? v : vn;
            const uint64_t T = delta >= 63 ? 0 : (lo + (hi << 16)) >> delta;
            if (mine) {
                st.acc[n][t][2 * r] = (int)(upper ? (T >> 16) & 0xFFu : T & 0xFFu);
                st.acc[n][t][2 * r + 1] = (int)(upper ? (T >> 24) : (T >> 8) & 0xFFu);
            }
        }
}

// One warp consumes its 32 keys (kw .. kw + 31) of a tile on the tensor-core
// path.  RES = false: binary-only keys (a binary cache, or the adaptive
// cache's second segment): no residual score, the sign part alone.
// BM: the binary row map, for binary-only keys (a binary cache, or the
// adaptive cache's binary-only segment), whose rows need not line up with
// the codes': row tile 8w + t = sign bit t of bytes 16w + g8 / 16w + g8 + 8
// of sign window w, 2^t units per unit (one mask per fragment instead of a
// shift and a mask).  Not at head_dim 64, whose fragments hold one sign byte
// per row pair.
template <int D, int GC, typename Cfg, bool ENT = false, bool RES = true, bool BM = false, int NRT = 8>
__device__ __forceinline__ void consume_warp_tile_mma(const QSmem& qs, MmaState<GC, NRT>& st, const uint8_t* sb,
                                                      int kw, int nk, uint8_t* wb, int* dotb) {
    static_assert(nib_by_bit(D) && NRT == D / 16, "tensor-core path: head dims 64, 128, 256");
    static_assert(!(BM && RES) && !(BM && D == 64), "the binary row map: no codes, not at head_dim 64");
    constexpr int NT = MmaState<GC, NRT>::NT, NWD = D / 32;
    constexpr int WB_PART = 8 * NT * Cfg::WB_ROW;
    const int lane = threadIdx.x & 31;
    const int kk = kw + lane;
    const bool valid = kk < nk;
    if constexpr (RES) {
        residual_dots_mma<D, GC>(sb + Cfg::OFF_KNIB, kw, qs.qa, dotb);
        __syncwarp();
    }
    // ---- score phase: lane `lane` scores key kk for the GC heads ----------------
    uint32_t ks[NWD];
    if constexpr (NWD == 2) {
        const uint2 v = *reinterpret_cast<const uint2*>(sb + Cfg::OFF_KSIGN + kk * (D / 8));
        ks[0] = v.x;
        ks[1] = v.y;
    } else {
#pragma unroll
        for (int c = 0; c < NWD / 4; ++c) {
            const uint4 v = *reinterpret_cast<const uint4*>(sb + Cfg::OFF_KSIGN + kk * (D / 8) + 16 * c);
            ks[4 * c] = v.x;
            ks[4 * c + 1] = v.y;
            ks[4 * c + 2] = v.z;
            ks[4 * c + 3] = v.w;
        }
    }
    const float kbs = __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_KBS)[kk]);
    const float krs = RES ? __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_KRS)[kk]) : 0.0f;
    float s2[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        const float4 cst = *reinterpret_cast<const float4*>(qs.c + 4 * g);  // bco, rco, off8, eco
        int pop = 0;
#pragma unroll
        for (int k = 0; k < NWD; ++k) pop += __popc(qs.sign[8 * g + k] ^ ks[k]);
        float s = cst.x * kbs * (float)(D - 2 * pop);
        if (RES) s = fmaf(cst.y * krs, (float)(dotb[g * kDotRow + lane] - __float_as_int(cst.z)), s);
        s2[g] = valid ? s : -INFINITY;
        if constexpr (ENT) {
            // xnor_dot without 1/sqrt(d), online per lane (adaptive_precision.cu:69-102)
            if (valid) {
                const float sc = cst.w * kbs * (float)(D - 2 * pop);
                if (sc > st.em[g]) {
                    const float f = (st.em[g] == -INFINITY) ? 0.0f : __expf(st.em[g] - sc);
                    st.ez[g] = st.ez[g] * f + 1.0f;
                    st.ew[g] = st.ew[g] * f + sc;
                    st.em[g] = sc;
                } else {
                    const float e = __expf(sc - st.em[g]);
                    st.ez[g] += e;
                    st.ew[g] += e * sc;
                }
            }
        }
    }
    const float vbs = valid ? __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_VBS)[kk]) : 0.0f;
    const float vrs = (RES && valid) ? __half2float(reinterpret_cast<const __half*>(sb + Cfg::OFF_VRS)[kk]) : 0.0f;
    // per-key weight multipliers: sign coefficient 2 bscale, code coefficient
    // rscale / 7, constant term bscale + 8 rscale / 7 (bits {0,1} and codes + 8)
    const float cs = 2.0f * vbs, cc = vrs * (1.0f / 7.0f), ct = vbs + 8.0f * cc;
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        // e = 2^(s - U): the key's softmax weight in units of 2^U (while U is
        // unset, Uf = -inf makes every valid e infinite and forces the choice)
        float e = valid ? fast_exp2(s2[g] - st.Uf[g]) : 0.0f;
        float xa = e * cs, xr = e * cc;
        if (__any_sync(0xffffffffu, fmaxf(fmaxf(xa, xr), e * 0x1p-33f) >= 2147483648.0f)) {
            // New unit (warp-uniform, rare after the first tile): the warp's
            // largest coefficient lands in (2^21, 2^22] and every e below 2^62.
            // A raise by delta divides the accumulators and l, t by 2^delta.
            // (the floor 2^-40: keys whose coefficients are ~0 still bound e)
            float lg = valid ? s2[g] + log2f(fmaxf(fmaxf(cs, cc), 0x1p-40f)) : -INFINITY;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) lg = fmaxf(lg, __shfl_xor_sync(0xffffffffu, lg, off));
            if (lg > -INFINITY) {
                int Un = (int)ceilf(lg) - 22;
                if (st.U[g] != kUUnset) {
                    Un = max(Un, st.U[g] + 1);
                    const int delta = Un - st.U[g];
                    mma_shift_down(st, g, delta);
                    const float down = delta > 126 ? 0.0f : exp2i(-delta);
                    st.l[g] *= down;
                    st.t[g] *= down;
                }
                st.U[g] = Un;
                st.Uf[g] = (float)Un;
                e = valid ? fast_exp2(s2[g] - st.Uf[g]) : 0.0f;
                xa = e * cs;
                xr = e * cc;
            }
        }
        st.l[g] += e;
        st.t[g] = fmaf(e, ct, st.t[g]);
        const uint32_t A = __float2uint_rn(xa), R = __float2uint_rn(xr);
        // head_dim 64: the sign fragments' k index of key `lane` (see above)
        const int sign_k = (D == 64) ? ((lane & 1) ? 16 : 0) + 4 * (lane >> 3) + ((lane & 7) >> 1) : lane;
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            wb[(4 * g + n) * Cfg::WB_ROW + sign_k] = (uint8_t)(A >> (8 * n));
            if (RES) wb[WB_PART + (4 * g + n) * Cfg::WB_ROW + lane] = (uint8_t)(R >> (8 * n));
        }
    }
    __syncwarp();
    const int g8 = lane >> 2, q = lane & 3;
    uint32_t bs[NT][2], br[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const bool ok = 8 * n + g8 < 4 * GC;
        const uint8_t* rs = wb + (8 * n + g8) * Cfg::WB_ROW + 4 * q;
        bs[n][0] = ok ? *reinterpret_cast<const uint32_t*>(rs) : 0u;
        bs[n][1] = ok ? *reinterpret_cast<const uint32_t*>(rs + 16) : 0u;
        br[n][0] = (RES && ok) ? *reinterpret_cast<const uint32_t*>(rs + WB_PART) : 0u;
        br[n][1] = (RES && ok) ? *reinterpret_cast<const uint32_t*>(rs + WB_PART + 16) : 0u;
    }
    // ---- sign part: bits c and c + 4 of sign bytes g8, g8 + 8 -------------------
    if constexpr (BM) {  // binary row map: tile 8w + t = bit t of sign bytes 16w + g8, 16w + g8 + 8
#pragma unroll
        for (int w = 0; w < D / 128; ++w) {
            uint32_t r0, r1, r2, r3;
            ldsm_x2_trans_b8(sb + Cfg::OFF_VSIGN + kk * (D / 8) + 16 * w, r0, r1, r2, r3);
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const uint32_t mk = 0x01010101u << t;
#pragma unroll
                for (int n = 0; n < NT; ++n)
                    mma_u8(st.acc[n][8 * w + t], r0 & mk, r1 & mk, r2 & mk, r3 & mk, bs[n][0], bs[n][1]);
            }
        }
    } else if constexpr (D == 64) {  // tile t: bits t, t + 4 of sign byte g8; keys in sign_k order
        uint32_t r0, r1;
        ldsm_x1_trans_b8(sb + Cfg::OFF_VSIGN + kw * (D / 8) + 16 * (lane & 15), r0, r1);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t s0 = r0 >> t, s1 = r1 >> t;
#pragma unroll
            for (int n = 0; n < NT; ++n)
                mma_u8(st.acc[n][t], s0 & 0x01010101u, s0 & 0x10101010u, s1 & 0x01010101u, s1 & 0x10101010u,
                       bs[n][0], bs[n][1]);
        }
    } else {
#pragma unroll
        for (int w = 0; w < D / 128; ++w) {  // 16-byte window w of the sign row: tiles 8w ..
            uint32_t r0, r1, r2, r3;
            ldsm_x2_trans_b8(sb + Cfg::OFF_VSIGN + kk * (D / 8) + 16 * w, r0, r1, r2, r3);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t s0 = r0 >> c, s1 = r1 >> c, s2b = r2 >> c, s3 = r3 >> c;
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    mma_u8(st.acc[n][8 * w + 2 * c], s0 & 0x01010101u, s0 & 0x10101010u, s2b & 0x01010101u,
                           s2b & 0x10101010u, bs[n][0], bs[n][1]);
                    mma_u8(st.acc[n][8 * w + 2 * c + 1], s1 & 0x01010101u, s1 & 0x10101010u, s3 & 0x01010101u,
                           s3 & 0x10101010u, bs[n][0], bs[n][1]);
                }
            }
        }
    }
    // ---- residual part: nibble chunk c, bytes g8, g8 + 8 --------------------------
    if constexpr (RES) {
        const uint8_t* vn = sb + Cfg::OFF_VNIB + (kk >> 3) * (4 * D) + 16 * (kk & 7);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
            uint32_t r0, r1, r2, r3;
            ldsm_x2_trans_b8(vn + 128 * c, r0, r1, r2, r3);
            // row tiles of the chunk's bytes g8 and g8 + 8: 2c, 2c + 1 (head_dim 64:
            // chunk c holds tiles 2c, 2c + 1 as its two byte halves); head_dim 256:
            // window c / 4, tiles 8 (c / 4) + 2 (c % 4) (+ 1)
            const int t0 = (D == 256) ? 8 * (c >> 2) + 2 * (c & 3) : 2 * c;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                mma_u8(st.acc[n][t0], r0 & 0x0F0F0F0Fu, r0 & 0xF0F0F0F0u, r2 & 0x0F0F0F0Fu, r2 & 0xF0F0F0F0u,
                       br[n][0], br[n][1]);
                mma_u8(st.acc[n][t0 + 1], r1 & 0x0F0F0F0Fu, r1 & 0xF0F0F0F0u, r3 & 0x0F0F0F0Fu, r3 & 0xF0F0F0F0u,
                       br[n][0], br[n][1]);
            }
        }
    }
    __syncwarp();  // the scratch is rewritten by the next tile
}

// Entropy partials (max, sum e^(s-max), sum e^(s-max) s) merge by the
// log-sum-exp rule; H = log z + max - w / max(z, 1e-12) (adaptive_precision.cu:120-128).
struct EntPart {
    float m, z, w;
};

__device__ __forceinline__ EntPart ent_merge(EntPart a, EntPart b) {
    const float M = fmaxf(a.m, b.m);
    if (M == -INFINITY) return a;
    const float fa = (a.m == -INFINITY) ? 0.0f : __expf(a.m - M);
    const float fb = (b.m == -INFINITY) ? 0.0f : __expf(b.m - M);
    return EntPart{M, a.z * fa + b.z * fb, a.w * fa + b.w * fb};
}

__device__ __forceinline__ float ent_value(EntPart t) { return logf(t.z) + t.m - t.w / fmaxf(t.z, 1e-12f); }

// Final (m in log2 units, l, o) of head h, dim i: to the outputs, or in an
// exchange to this rank's slot of every rank's buffer (natural-log m).
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// One exchange word: the value's bits low, the call epoch high.  A single
// aligned 64-bit access is indivisible, so a reader that sees the epoch sees
// the value with it: no fence or separate flag is needed.
__device__ __forceinline__ unsigned long long xword(float v, unsigned epoch) {
    return ((unsigned long long)epoch << 32) | __float_as_uint(v);
}

template <int D>
__device__ __forceinline__ void emit_final(const DecodeArgs& a, int64_t h, int i, float M, float L, float O) {
    if (a.xw > 0) {
        const int64_t n_heads = (int64_t)a.n_slots * a.group;
        const int64_t off = (((int64_t)(a.xepoch & 1u) * a.xw + a.xrank) * n_heads + h) * (D + 2);
        const unsigned long long wo = xword(O, a.xepoch), wm = xword(M * kLn2, a.xepoch), wl = xword(L, a.xepoch);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j >= a.xw) break;
            unsigned long long* p = a.xparts[j] + off;
            if (i == 0) {
                st_relaxed_sys_u64(p, wm);
                st_relaxed_sys_u64(p + 1, wl);
            }
            st_relaxed_sys_u64(p + 2 + i, wo);
        }
        return;
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

// Exchange epilogue of a (slot, head group): every thread waits (bounded) for
// the words of its dims from every rank in this rank's buffer, then merges
// the xw partials.  Words carry the call's epoch and are compared as "at
// least"; partials alternate between two parity halves, so a rank that is a
// step ahead writes the other half and never overwrites data still read.
template <int D, int GC>
__device__ __forceinline__ void xchg_finish(const DecodeArgs& a, int slot, int hg) {
    const int tid = threadIdx.x;
    const int64_t n_heads = (int64_t)a.n_slots * a.group;
    const int64_t head0 = (int64_t)slot * a.group + (int64_t)hg * GC;
    const unsigned long long* base = a.xparts[a.xrank] + (int64_t)(a.xepoch & 1u) * a.xw * n_heads * (D + 2);
    __shared__ int s_timeout;
    if (tid == 0) s_timeout = 0;
    __syncthreads();
    volatile int* gave_up = &s_timeout;
    // A word already loaded once (v), polled again at most a.xspin times
    // (after 4096 fast polls with 256 ns sleeps) while it carries an older
    // epoch.  Once any thread of the CTA has given up, every other poll
    // returns at once, so a missing rank costs one spin limit per CTA, not
    // one per word.
    auto settle = [&](unsigned long long v, const unsigned long long* p) -> float {
        for (uint32_t it = 0; (int)((unsigned)(v >> 32) - a.xepoch) < 0; ++it) {
            if (it >= a.xspin || *gave_up) {
                *gave_up = 1;
                return 0.0f;
            }
            if (it >= 4096) __nanosleep(256);  // back off only after a few microseconds
            v = ld_relaxed_sys_u64(p);
        }
        return __uint_as_float((unsigned)v);
    };
    for (int idx = tid; idx < GC * D; idx += kDecThreads) {
        const int g = idx / D, i = idx % D;
        const int64_t h = head0 + g;
        // all 3 xw words first, so that their loads are in flight together
        // (one round trip, not 3 xw); then only the words that do not yet
        // carry this call's epoch are polled again
        unsigned long long w[8][3];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j >= a.xw) break;
            const unsigned long long* r = base + ((int64_t)j * n_heads + h) * (D + 2);
            w[j][0] = ld_relaxed_sys_u64(r);
            w[j][1] = ld_relaxed_sys_u64(r + 1);
            w[j][2] = ld_relaxed_sys_u64(r + 2 + i);
        }
        float mj[8], lj[8], oj[8];
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j >= a.xw) break;
            const unsigned long long* r = base + ((int64_t)j * n_heads + h) * (D + 2);
            mj[j] = settle(w[j][0], r);
            lj[j] = settle(w[j][1], r + 1);
            oj[j] = settle(w[j][2], r + 2 + i);
            if (lj[j] > 0.0f) M = fmaxf(M, mj[j]);
        }
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j >= a.xw) break;
            if (lj[j] > 0.0f) {
                const float f = __expf(mj[j] - M);
                L += lj[j] * f;
                O += oj[j] * f;
            }
        }
        if (a.out) a.out[h * D + i] = __float2half((L > 0.0f) ? O * (1.0f / L) : 0.0f);
    }
    __syncthreads();
    if (tid == 0 && s_timeout) raise_device_error(&g_bc_device_error, BC_DEVERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// End of a CTA: reduce each warp, merge the warps (log-sum-exp), then either
// write the outputs (single split) or publish a partial and let the last CTA
// of the (slot, head group) combine all splits.
// ---------------------------------------------------------------------------
// Per-warp record (m, l, o[d] - t) of each head into mg[warp][g][d + 2]:
// f32x2 accumulators, reduced over the lanes holding the same dims.
template <int D, int GC, typename Cfg>
__device__ __forceinline__ void warp_records(float* mg, SoftState<GC, Cfg::NP>& st, bool /*bm*/) {
    constexpr int KPW = Cfg::KPW, DL = Cfg::DL, NP = Cfg::NP;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, qt = lane / KPW;
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        float l = st.l[g], t = st.t[g];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            l += __shfl_xor_sync(0xffffffffu, l, off);
            t += __shfl_xor_sync(0xffffffffu, t, off);
        }
        float o[DL];
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const float fs = exp2i(kAccShift - p);
            const float fn = exp2i(kAccShift - 4 * (p & 3));
            o[p] = st.acc_s[g][p].x * fs + st.acc_n[g][p].x * fn;
            o[p + NP] = st.acc_s[g][p].y * fs + st.acc_n[g][p].y * fn;
        }
        // lanes holding the same chunk (same qt) differ in their low log2(KPW) bits
#pragma unroll
        for (int off = 1; off < KPW; off <<= 1)
#pragma unroll
            for (int i = 0; i < DL; ++i) o[i] += __shfl_xor_sync(0xffffffffu, o[i], off);
        float* rec = mg + ((size_t)warp * GC + g) * (D + 2);
        if (lane % KPW == 0) {
#pragma unroll
            for (int i = 0; i < DL; ++i) rec[2 + DL * qt + i] = o[i] - t;
        }
        if (lane == 0) {
            rec[0] = st.m[g];
            rec[1] = l;
        }
    }
}

// The same record from the tensor-core accumulators.  Each lane dumps its
// fragments to shared memory (the ring is free by now); lane l then takes dims
// (D / 32) l .. of every head: dim = 128 w + 64 h + 8 g8 + c + 4 hi sits in row
// tile 8 w + 2c + h (head_dim 64: tile c + 2 h', dim = 8 g8 + 2 h' + c' + 4 hi,
// i.e. tile dim % 4), row g8 + 8 hi (16 units per unit when hi), column tile
// g / 2, byte columns 0-1 in lane 4 g8 + 2 (g % 2) and 2-3 in the lane after it.
// bm: the accumulators were filled with the binary row map (dim = 128 w +
// 64 h + 8 g8 + t in tile 8 w + t, row g8 + 8 h, 2^t units per unit).
template <int D, int GC, typename Cfg, int NRT>
__device__ __forceinline__ void warp_records(float* mg, MmaState<GC, NRT>& st, bool bm) {
    constexpr int NT = MmaState<GC, NRT>::NT, DS = Cfg::DUMP_STRIDE;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int* dump = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(mg) + Cfg::DUMP_OFF) + warp * 32 * DS;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int t = 0; t < NRT; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) dump[lane * DS + 4 * NRT * n + 4 * t + i] = st.acc[n][t][i];
    __syncwarp();
#pragma unroll
    for (int g = 0; g < GC; ++g) {
        float l = st.l[g], t = st.t[g];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            l += __shfl_xor_sync(0xffffffffu, l, off);
            t += __shfl_xor_sync(0xffffffffu, t, off);
        }
        float* rec = mg + ((size_t)warp * GC + g) * (D + 2);
        // l, t and the accumulators are all in units of 2^U: U is the record's
        // reference point (log2), -inf when the warp saw no key
        if (lane == 0) {
            rec[0] = st.Uf[g];
            rec[1] = l;
        }
#pragma unroll
        for (int e = 0; e < D / 32; ++e) {
            const int dim = (D / 32) * lane + e;
            const int h = (dim >> 6) & 1, w = dim >> 7, g8 = (dim >> 3) & 7, c = dim & 3, hi = (dim >> 2) & 1;
            // shared map: tile 8w + 2c + h (head_dim 64: tile c), row g8 + 8 hi;
            // binary map: tile 8w + dim % 8, row g8 + 8 h
            const int tile = bm ? 8 * w + (dim & 7) : (D == 64 ? c : 8 * w + 2 * c + h), upper = bm ? h : hi;
            const int* la = dump + (4 * g8 + 2 * (g & 1)) * DS + 4 * NRT * (g >> 1) + 4 * tile + 2 * upper;
            const int* lb = la + DS;
            const uint64_t v0 = (uint64_t)(uint32_t)la[0] + ((uint64_t)(uint32_t)la[1] << 8);
            const uint64_t v1 = (uint64_t)(uint32_t)lb[0] + ((uint64_t)(uint32_t)lb[1] << 8);
            const float unit = bm ? exp2i(-(dim & 7)) : (hi ? (1.0f / 16.0f) : 1.0f);
            const float v = ((float)v0 + 65536.0f * (float)v1) * unit;
            rec[2 + dim] = v - t;
        }
    }
}

template <int D, int GC, typename Cfg, bool ENT = false, typename St>
__device__ __forceinline__ void finish_cta(const DecodeArgs& a, int slot, int hg, int split, uint8_t* smem, St& st,
                                           bool bm = false) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __syncthreads();  // ring no longer in use
    float* mg = reinterpret_cast<float*>(smem);  // [warps][GC][D+2]
    warp_records<D, GC, Cfg>(mg, st, bm);
    __shared__ EntPart s_ent[ENT ? kWarps : 1][ENT ? GC : 1];
    if constexpr (ENT) {
#pragma unroll
        for (int g = 0; g < GC; ++g) {
            EntPart e{st.em[g], st.ez[g], st.ew[g]};
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
                e = ent_merge(e, EntPart{__shfl_xor_sync(0xffffffffu, e.m, off), __shfl_xor_sync(0xffffffffu, e.z, off),
                                         __shfl_xor_sync(0xffffffffu, e.w, off)});
            if (lane == 0) s_ent[warp][g] = e;
        }
    }
    __syncthreads();
    const bool single = (a.n_splits == 1);
    const int64_t head0 = (int64_t)slot * a.group + (int64_t)hg * GC;
    if constexpr (ENT) {
        if (tid < GC) {
            EntPart e = s_ent[0][tid];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) e = ent_merge(e, s_ent[w][tid]);
            const int64_t h = head0 + tid;
            if (single) {
                a.entropy[h] = ent_value(e);
            } else {
                float* p = a.ws_ent + (h * a.n_splits + split) * 3;
                p[0] = e.m;
                p[1] = e.z;
                p[2] = e.w;
            }
        }
    }
    for (int idx = tid; idx < GC * D; idx += kDecThreads) {
        const int g = idx / D, i = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mg[((size_t)w * GC + g) * (D + 2)]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float* rec = mg + ((size_t)w * GC + g) * (D + 2);
            const float f = (rec[0] == -INFINITY) ? 0.0f : fast_exp2(rec[0] - M);
            L += rec[1] * f;
            O += rec[2 + i] * f;
        }
        const int64_t h = head0 + g;
        if (single) {
            emit_final<D>(a, h, i, M, L, O);
        } else {
            float* p = a.ws_part + (h * a.n_splits + split) * (D + 4);
            if (i == 0) {
                p[0] = M;
                p[1] = L;
            }
            p[4 + i] = O;
        }
    }
    if (single) {
        if (a.xw > 0) xchg_finish<D, GC>(a, slot, hg);
        return;
    }
    __shared__ unsigned s_last;
    __syncthreads();
    if (tid == 0) {
        // acq_rel at GPU scope, instead of fences around a plain atomic: it
        // releases this CTA's partial (written by all threads, ordered before
        // this one by the barrier above) and, in the last CTA, acquires every
        // other CTA's; the barrier below extends that to all its threads.
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(&a.ws_cnt[(int64_t)slot * a.n_hgroups + hg])
                     : "memory");
        s_last = (prev == (unsigned)(a.n_splits - 1)) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    // Split combine.  A task is (head, 4 dims); the threads left over split
    // the splits into SG interleaved groups, so several L2 round trips run in
    // parallel.  Each thread loads kComb partials at once (m, l, float4 of o),
    // merges them into a running (M, L, O), and the SG group results are then
    // merged through shared memory (the ring, free by now).
    constexpr int kComb = BC_DEC_KCOMB;
    constexpr int TASKS = GC * D / 4;
    constexpr int SG = (TASKS >= kDecThreads) ? 1 : kDecThreads / TASKS;
    float* cmb = reinterpret_cast<float*>(smem);  // [SG][TASKS][6]
    static_assert(SG * TASKS * 6 * 4 <= Cfg::BODY_B, "combine scratch exceeds the ring");
    for (int t = tid; t < TASKS * SG; t += kDecThreads) {
        const int task = t % TASKS, sg = t / TASKS;
        const int g = task / (D / 4), c = task % (D / 4);
        const int64_t h = head0 + g;
        const float* base = a.ws_part + h * a.n_splits * (D + 4);
        float M = -INFINITY, L = 0.0f;
        float4 O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int j0 = sg * kComb; j0 < a.n_splits; j0 += SG * kComb) {
            float mj[kComb], lj[kComb];
            float4 oj[kComb];
#pragma unroll
            for (int k = 0; k < kComb; ++k) {
                const bool in = j0 + k < a.n_splits;
                const float* r = base + (size_t)(j0 + k) * (D + 4);
                mj[k] = in ? __ldcg(r) : -INFINITY;
                lj[k] = in ? __ldcg(r + 1) : 0.0f;
                oj[k] = in ? __ldcg(reinterpret_cast<const float4*>(r + 4) + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            float Mn = M;
#pragma unroll
            for (int k = 0; k < kComb; ++k) Mn = fmaxf(Mn, mj[k]);
            const float fo = (M == -INFINITY) ? 0.0f : fast_exp2(M - Mn);
            L *= fo;
            O.x *= fo; O.y *= fo; O.z *= fo; O.w *= fo;
#pragma unroll
            for (int k = 0; k < kComb; ++k) {
                const float f = (mj[k] == -INFINITY) ? 0.0f : fast_exp2(mj[k] - Mn);
                L += lj[k] * f;
                O.x += oj[k].x * f; O.y += oj[k].y * f; O.z += oj[k].z * f; O.w += oj[k].w * f;
            }
            M = Mn;
        }
        float* e = cmb + (sg * TASKS + task) * 6;
        e[0] = M; e[1] = L; e[2] = O.x; e[3] = O.y; e[4] = O.z; e[5] = O.w;
    }
    __syncthreads();
    for (int idx = tid; idx < GC * D; idx += kDecThreads) {
        const int task = idx >> 2, k = idx & 3;
        const int64_t h = head0 + task / (D / 4);
        float M = -INFINITY;
#pragma unroll
        for (int sg = 0; sg < SG; ++sg) M = fmaxf(M, cmb[(sg * TASKS + task) * 6]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int sg = 0; sg < SG; ++sg) {
            const float* e = cmb + (sg * TASKS + task) * 6;
            const float f = (e[0] == -INFINITY) ? 0.0f : fast_exp2(e[0] - M);
            L += e[1] * f;
            O += e[2 + k] * f;
        }
        emit_final<D>(a, h, idx % D, M, L, O);
    }
    if constexpr (ENT) {
        if (tid < GC) {
            const int64_t h = head0 + tid;
            const float* base = a.ws_ent + h * a.n_splits * 3;
            EntPart e{-INFINITY, 0.0f, 0.0f};
            for (int j = 0; j < a.n_splits; ++j)
                e = ent_merge(e, EntPart{__ldcg(base + 3 * j), __ldcg(base + 3 * j + 1), __ldcg(base + 3 * j + 2)});
            a.entropy[h] = ent_value(e);
        }
    }
    if (tid == 0) a.ws_cnt[(int64_t)slot * a.n_hgroups + hg] = 0u;  // leave the counter zeroed
    if (a.xw > 0) xchg_finish<D, GC>(a, slot, hg);
}

__device__ __forceinline__ void cta_coords(const DecodeArgs& a, int& slot, int& hg, int& split) {
    const int cta = blockIdx.x;
    split = cta % a.n_splits;
    const int rest = cta / a.n_splits;
    hg = rest % a.n_hgroups;
    slot = rest / a.n_hgroups;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------
// Fused decode step helpers.  The CTAs whose key range holds the append
// position encode the new K (warp 0) and V (warp 1) row with the shared
// warp encoders (bit-identical to bc_append_kv), stage it in shared memory,
// and, in head group 0 only, store it to the planes.  When the tile holding
// that position lands, its owning warp overwrites the stale row in the stage
// before scoring, so the tile is attended exactly as if the append had run
// first, whatever the ring copy read from global memory.
// ---------------------------------------------------------------------------
template <int NW>
struct StagedRowSink {
    PlaneRowSink<NW> g;  // global row (written when `store`)
    uint8_t* srow;       // shared-memory row: sign words, nibble chunks, scales
    int nib_off;
    bool store;
    __device__ __forceinline__ void sign(const uint32_t (&w)[NW], int lane) {
        if (store) g.sign(w, lane);
#pragma unroll
        for (int k = 0; k < NW; ++k)
            if (lane == k) reinterpret_cast<uint32_t*>(srow)[k] = w[k];
    }
    __device__ __forceinline__ void bscale(uint16_t b) {
        if (store) g.bscale(b);
        reinterpret_cast<uint16_t*>(srow + nib_off + 16 * NW)[0] = b;
    }
    __device__ __forceinline__ void nib(const uint32_t (&nw)[NW], int lane) {
        if (store) g.nib(nw, lane);
        if constexpr (nib_by_bit(32 * NW)) {  // lanes L < 4 hold the row's words (staged chunks 16 B apart)
            if (lane < 4) nib_words_to<NW>(srow + nib_off, 16, nw, lane);
        } else {
#pragma unroll
            for (int k = 0; k < NW; ++k)
                if ((lane & 7) == 0)
                    reinterpret_cast<uint32_t*>(srow + nib_off + 16 * k)[lane >> 3] = nw[k] ^ 0x88888888u;
        }
    }
    __device__ __forceinline__ void rscale(uint16_t b) {
        if (store) g.rscale(b);
        reinterpret_cast<uint16_t*>(srow + nib_off + 16 * NW)[1] = b;
    }
};

template <int D, typename Cfg>
// Arguments by value: a reference to the kernel's parameter block would
// make the compiler copy that block to the stack of every thread.
__device__ __noinline__ void encode_append_row(const __half* src, bc_kv_planes P, int64_t row, bool store,
                                               int append_res, int head_dim, uint8_t* smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;  // warp 0: K, warp 1: V
    uint8_t* srow = smem + Cfg::NEW_OFF + warp * Cfg::NEWROW_B;
    if (append_res == BC_RES_NONE) {
        // binary append: the staged residual is code 0 (offset-binary 0x8) with scale 0
        if (lane < D / 8) reinterpret_cast<uint32_t*>(srow + Cfg::NEWSIGN_B)[lane] = 0x88888888u;
        if (lane == 0) reinterpret_cast<uint16_t*>(srow + Cfg::NEWSIGN_B + D / 2)[1] = 0;
    }
    float x[D / 32];
    load_vec<D / 32>(src, lane, x);
    if (row < 0) {
        if (store && lane == 0) raise_device_error(&g_bc_device_error, BC_DEVERR_PAGE);
        store = false;  // attend the staged row, store nothing
    }
    StagedRowSink<D / 32> sink{{P, row}, srow, Cfg::NEWSIGN_B, store};
    switch (append_res) {
        case BC_RES_NONE: encode_row<D / 32, BC_RES_NONE>(x, lane, head_dim, sink); break;
        case BC_RES_FP16_SCALE: encode_row<D / 32, BC_RES_FP16_SCALE>(x, lane, head_dim, sink); break;
        default: encode_row<D / 32, BC_RES_FP32_SCALE>(x, lane, head_dim, sink); break;
    }
}

// Overwrite key kk of a landed stage with the staged rows (one warp).
template <int D, bool COMP, typename Cfg>
__device__ __forceinline__ void patch_stage_row(uint8_t* sb, int kk, const uint8_t* smem) {
    constexpr int NWD = D / 32;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint8_t* srow = smem + Cfg::NEW_OFF + j * Cfg::NEWROW_B;
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(srow + Cfg::NEWSIGN_B + D / 2);
        const int off_sign = j ? Cfg::OFF_VSIGN : Cfg::OFF_KSIGN, off_bs = j ? Cfg::OFF_VBS : Cfg::OFF_KBS;
        if (lane < NWD)
            reinterpret_cast<uint32_t*>(sb + off_sign)[kk * NWD + lane] = reinterpret_cast<const uint32_t*>(srow)[lane];
        if (lane == 0) reinterpret_cast<uint16_t*>(sb + off_bs)[kk] = sc[0];
        if (COMP) {
            const int off_nib = j ? Cfg::OFF_VNIB : Cfg::OFF_KNIB, off_rs = j ? Cfg::OFF_VRS : Cfg::OFF_KRS;
            if (lane < NWD)
                *reinterpret_cast<uint4*>(sb + off_nib + nib_chunk_offset(kk, lane, D)) =
                    reinterpret_cast<const uint4*>(srow + Cfg::NEWSIGN_B)[lane];
            if (lane == 0) reinterpret_cast<uint16_t*>(sb + off_rs)[kk] = sc[1];
        }
    }
    // the stage is refilled by the async proxy later: order these writes first
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
}

// Stage layout of the adaptive kernel's binary-only segment on the tensor-core
// path: four 128-key tiles per ring stage (sign words and scales only, 18 KB
// at head_dim 128, 10 KB at 64, 34 KB at 256), so a binary CTA keeps four
// times the bytes in flight.
template <int D>
struct BinStageCfg {
    static constexpr int NWD = D / 32;
    static constexpr int TILES = 4;
    static constexpr int KEYS = TILES * kTile;
    static constexpr int OFF_KSIGN = 0;
    static constexpr int OFF_KBS = OFF_KSIGN + KEYS * D / 8;
    static constexpr int OFF_VSIGN = OFF_KBS + KEYS * 2;
    static constexpr int OFF_VBS = OFF_VSIGN + KEYS * D / 8;
    static constexpr int BYTES = OFF_VBS + KEYS * 2;
    static constexpr int OFF_KNIB = 0, OFF_KRS = 0, OFF_VNIB = 0, OFF_VRS = 0;  // no residual planes
    static constexpr int WB_ROW = DecCfg<D, 1, true>::WB_ROW;
};

// ---------------------------------------------------------------------------
// Plane-layout kernel.  Thread 0 keeps the ring full: at iteration `it` it
// refills the stage consumed at iteration it-LAG once all four warps have
// released it (per-stage "empty" mbarrier, one arrival per warp).  Warps
// otherwise run free: no CTA-wide barrier per tile.
// ---------------------------------------------------------------------------
// VAR: 0 attention, 1 fused decode step (append + attend, paged caches),
// 2 attention plus the per-head entropy of the binary-score softmax,
// 3 attention over a compact adaptive cache (compensated keys, then
// binary-only keys; instantiated with COMP = true).
template <int D, int GC, bool COMP, int VAR = 0>
__global__ void __launch_bounds__(kDecThreads, DecCfg<D, GC, COMP>::MIN_CTAS)
    k_decode_planes(const DecodeArgs a) {
    constexpr bool STEP = VAR == 1, ENT = VAR == 2, ADA = VAR == 3;
    using Cfg = DecCfg<D, GC, COMP>;
    static_assert(Cfg::MMA || !COMP || !nib_by_bit(D),
                  "compensated planes in the by-bit nibble order need the tensor-core path");
    constexpr int NS = Cfg::NS, LAG = Cfg::LAG, T = Cfg::T;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = aligned_smem(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int slot, hg, split;
    cta_coords(a, slot, hg, split);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::FULL_OFF);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + Cfg::EMPTY_OFF);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::FLAG_OFF);

    // adaptive caches: this CTA's segment (binary-only keys when seg_bin)
    const bool seg_bin = ADA && split >= a.nc;
    int s_begin, s_end;
    if constexpr (ADA) {
        if (seg_bin) {
            s_begin = (split - a.nc) * a.kps_bin;
            s_end = min(a.seq_len - a.n_keep, s_begin + a.kps_bin);
        } else {
            s_begin = split * a.keys_per_split;
            s_end = min(a.n_keep, s_begin + a.keys_per_split);
        }
    } else {
        s_begin = split * a.keys_per_split;
        s_end = min(a.seq_len, s_begin + a.keys_per_split);
    }
    const int n_keys = max(0, s_end - s_begin);
    // keys per ring stage: one tile, or four in the binary segment of the
    // adaptive kernel's tensor-core path
    constexpr bool BIN4 = ADA && Cfg::MMA;
    if constexpr (BIN4) static_assert(BinStageCfg<D>::BYTES <= Cfg::STAGE_B, "binary stage exceeds the ring stage");
    const bool wide = BIN4 && seg_bin;
    const int TS = wide ? BinStageCfg<D>::KEYS : ((VAR == 0 || VAR == 2) ? Cfg::KEYS : T);
    const int n_tiles = (n_keys + TS - 1) / TS;

    // fused step: does this CTA's key range hold the append position?
    const bool appends = STEP && a.append_pos >= s_begin && a.append_pos < s_end;
    const __half* new_src[2] = {nullptr, nullptr};
    auto fetch_new_rows = [&]() {
        if constexpr (STEP) {
            if (appends) {
                const __half* g[2] = {a.new_k + (int64_t)slot * D, a.new_v + (int64_t)slot * D};
                const bool aligned = ((reinterpret_cast<uintptr_t>(g[0]) | reinterpret_cast<uintptr_t>(g[1])) & 15) == 0;
                __half* raw = reinterpret_cast<__half*>(smem + Cfg::NEWRAW_OFF);
                for (int j = 0; j < 2; ++j) {
                    new_src[j] = aligned ? raw + j * D : g[j];
                    if (aligned)
                        for (int c = tid; c < D / 8; c += kDecThreads) cp_async16(raw + j * D + 8 * c, g[j] + 8 * c);
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
            }
        }
    };
    // Host-resident inputs are read before this kernel waits for the previous
    // one in the stream, so no earlier GPU work in the stream may write them
    // (the host synchronises before it rewrites them).  Their slow host-link
    // reads then overlap the previous kernel's tail.
    const bool q_host = STEP && (a.host_in & 1), kv_host = STEP && (a.host_in & 2);
    bool staged = false;
    if (q_host) staged = prefetch_query<D, GC, Cfg>(a, slot, hg, smem);
    if (kv_host) fetch_new_rows();
    // Launched with programmatic stream serialisation: everything above ran
    // while the previous kernel in the stream may still be finishing; wait
    // for it (and its memory) before the first access to device memory.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // Small inputs first: their copies start before the ring's bulk copies.
    if (!q_host) staged = prefetch_query<D, GC, Cfg>(a, slot, hg, smem);
    if (!kv_host) fetch_new_rows();

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // Plane row of a tile's first key.  Paged caches (the STEP variant only)
    // read the block table; tiles never straddle a page, since splits start on
    // tile boundaries and pages hold a multiple of the tile's 128 positions.
    auto row_of = [&](int tile) -> int64_t {
        if constexpr (STEP) return plane_row(a, slot, s_begin + tile * T);
        if constexpr (ADA) return (int64_t)slot * a.kv_stride + (seg_bin ? a.b0 : 0) + s_begin + (int64_t)tile * TS;
        return (int64_t)slot * a.kv_stride + s_begin + tile * T;
    };
    auto issue = [&](int tile, int stage, int64_t row) {
        const int k0 = tile * TS;
        const int nk = min(TS, n_keys - k0);
        const int nk8 = (nk + 7) & ~7;
        if constexpr (STEP) {
            if (row < 0) {
                // page id outside the pool: complete the stage without a copy and abort
                raise_device_error(&g_bc_device_error, BC_DEVERR_PAGE);
                *abort_flag = 1;
                mbar_arrive(&full[stage]);
                return;
            }
        }
        uint8_t* sbuf = smem + stage * Cfg::STAGE_B;
        const uint32_t sign_b = nk8 * (D / 8), sc_b = nk8 * 2, nib_b = nk8 * (D / 2);
        const bool res = COMP && !seg_bin;
        const uint32_t total = 2 * (sign_b + sc_b + (res ? nib_b + sc_b : 0));
        // residual planes: their own row stride in adaptive caches
        const int64_t rrow = ADA ? (int64_t)slot * a.res_stride + s_begin + k0 : row;
        mbar_arrive_expect_tx(&full[stage], total);
        using BS = BinStageCfg<D>;
        bulk_g2s(sbuf + (wide ? BS::OFF_KSIGN : Cfg::OFF_KSIGN), (const uint8_t*)a.K.sign + row * (D / 8), sign_b,
                 &full[stage]);
        bulk_g2s(sbuf + (wide ? BS::OFF_KBS : Cfg::OFF_KBS), (const uint8_t*)a.K.bscale + row * 2, sc_b, &full[stage]);
        bulk_g2s(sbuf + (wide ? BS::OFF_VSIGN : Cfg::OFF_VSIGN), (const uint8_t*)a.V.sign + row * (D / 8), sign_b,
                 &full[stage]);
        bulk_g2s(sbuf + (wide ? BS::OFF_VBS : Cfg::OFF_VBS), (const uint8_t*)a.V.bscale + row * 2, sc_b, &full[stage]);
        if (res) {
            bulk_g2s(sbuf + Cfg::OFF_KNIB, (const uint8_t*)a.K.nib + rrow * (D / 2), nib_b, &full[stage]);
            bulk_g2s(sbuf + Cfg::OFF_KRS, (const uint8_t*)a.K.rscale + rrow * 2, sc_b, &full[stage]);
            bulk_g2s(sbuf + Cfg::OFF_VNIB, (const uint8_t*)a.V.nib + rrow * (D / 2), nib_b, &full[stage]);
            bulk_g2s(sbuf + Cfg::OFF_VRS, (const uint8_t*)a.V.rscale + rrow * 2, sc_b, &full[stage]);
        }
    };
    // thread 0: the plane row of the next tile to issue, read one refill ahead
    // (a block-table load in paged caches)
    int64_t next_row = 0;
    if (tid == 0) {
        for (int t = 0; t < min(NS, n_tiles); ++t) issue(t, t, row_of(t));
        if (STEP && NS < n_tiles) next_row = row_of(NS);
    }

    QState<D, GC> qs;
    prepare_query<D, GC, COMP, Cfg, Cfg::MMA>(a, slot, hg, smem, qs, staged);
    const QSmem qsm{reinterpret_cast<const uint32_t*>(smem + Cfg::QSIGN_OFF),
                    reinterpret_cast<const float*>(smem + Cfg::QCONST_OFF), smem + Cfg::QPK_OFF};

    // Fused step: warps 0 and 1 encode the new K and V row; the owning warp
    // patches tile patch_it at key patch_kk (patch_it = -1: not this warp).
    int patch_it = -1, patch_kk = 0;
    if constexpr (STEP) {
        if (appends) {
            asm volatile("cp.async.wait_all;" ::: "memory");
            __syncthreads();
            if (warp < 2)
                encode_append_row<D, Cfg>(new_src[warp], warp == 0 ? a.K : a.V, plane_row(a, slot, a.append_pos),
                                          hg == 0, a.append_res, a.head_dim, smem);
            __syncthreads();
            const int rel = a.append_pos - s_begin;
            if ((rel % T) / 32 == warp) {
                patch_it = rel / T;
                patch_kk = rel % T;
            }
        }
    }
    // the tensor-core value phase (in adaptive caches the binary-only
    // segment runs its sign part alone)
    constexpr bool MMA = Cfg::MMA;
    std::conditional_t<MMA, MmaState<GC, Cfg::NRT>, SoftState<GC, Cfg::NP>> st;
    // the binary row map for binary-only keys: a binary cache, or the binary
    // segment of an adaptive cache (its CTAs see no code), not at head_dim 64
    constexpr bool BIN_BM = D != 64;
    const bool bm = Cfg::BM || (ADA && seg_bin && BIN_BM);
    init_soft(st);

    int it = 0;
    for (; it < n_tiles; ++it) {
        const int stage = it % NS;
        if (tid == 0 && it >= LAG && it - LAG + NS < n_tiles) {
            const int old = it - LAG;
            if (mbar_wait_bounded(&empty[old % NS], (uint32_t)(old / NS) & 1u)) {
                fence_proxy_async_smem();
                if constexpr (STEP) {
                    issue(old + NS, old % NS, next_row);
                    if (old + NS + 1 < n_tiles) next_row = row_of(old + NS + 1);
                } else {
                    issue(old + NS, old % NS, row_of(old + NS));
                }
            } else {
                *abort_flag = 1;
            }
        }
        bool ok = mbar_wait_bounded(&full[stage], (uint32_t)(it / NS) & 1u);
        if (!ok) *abort_flag = 1;
        if (*abort_flag) break;
        const int nk = min(TS, n_keys - it * TS);
        if constexpr (STEP) {
            if (it == patch_it) patch_stage_row<D, COMP, Cfg>(smem + stage * Cfg::STAGE_B, patch_kk, smem);
        }
        if constexpr (MMA) {
            uint8_t* wb = smem + Cfg::WB_OFF + warp * Cfg::WB_WARP;
            int* dotb = reinterpret_cast<int*>(smem + Cfg::DOT_OFF + warp * Cfg::DOT_WARP);
            uint8_t* sbuf = smem + stage * Cfg::STAGE_B;
            if (wide) {
                if constexpr (BIN4) {
                    for (int j = 0; j < BinStageCfg<D>::TILES && j * T < nk; ++j)
                        consume_warp_tile_mma<D, GC, BinStageCfg<D>, false, false, BIN_BM>(qsm, st, sbuf,
                                                                                           j * T + warp * 32, nk, wb,
                                                                                           dotb);
                }
            } else if (Cfg::TPS > 1 && TS > T) {
                for (int j = 0; j < Cfg::TPS && j * T < nk; ++j)
                    consume_warp_tile_mma<D, GC, Cfg, ENT, COMP, Cfg::BM>(qsm, st, sbuf, j * T + warp * 32, nk, wb, dotb);
            } else if (ADA && seg_bin)
                consume_warp_tile_mma<D, GC, Cfg, false, false, BIN_BM>(qsm, st, sbuf, warp * 32, nk, wb, dotb);
            else
                consume_warp_tile_mma<D, GC, Cfg, ENT, COMP, Cfg::BM>(qsm, st, sbuf, warp * 32, nk, wb, dotb);
        } else {
            if (ADA && seg_bin)
                consume_warp_tile<D, GC, false, Cfg>(qs, st, smem + stage * Cfg::STAGE_B, warp * 32, nk);
            else
                consume_warp_tile<D, GC, COMP, Cfg, ENT>(qs, st, smem + stage * Cfg::STAGE_B, warp * 32, nk);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
    }
    __syncthreads();
    // This CTA no longer needs the ring: let the next kernel in the stream be
    // scheduled as CTAs exit (it waits for this grid before touching memory).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (*abort_flag) {
        // A copy never landed (or a stage was never released): report, drain
        // what is still in flight (bounded), and leave.
        if (tid == 0) {
            raise_device_error(&g_bc_device_error, BC_DEVERR_TIMEOUT);
            const int issued = min(n_tiles, NS + max(0, it - LAG + 1));
            for (int t = max(0, it - NS); t < issued; ++t)
                mbar_wait_bounded(&full[t % NS], (uint32_t)(t / NS) & 1u);
        }
        return;
    }
    finish_cta<D, GC, Cfg, ENT>(a, slot, hg, split, smem, st, bm);
}

// ---------------------------------------------------------------------------
// Reference-record kernel: the same compute on tiles transcoded into the
// canonical shared-memory layout from BinaryVec (36 B) / ResidualVec (130 B,
// 2-byte aligned) arrays with plain loads.  K, V record bases are passed in
// .sign (BinaryVec*) and .nib (ResidualVec*); kv_stride = seq_len.
// ---------------------------------------------------------------------------
template <int D, bool COMP, typename Cfg>
__device__ __forceinline__ void load_tile_records(const DecodeArgs& a, int64_t rec0, int nk, uint8_t* sb) {
    constexpr int NWD = D / 32;
    const int kk = threadIdx.x;  // one key per thread (T == kDecThreads)
    if (kk >= nk) return;
    const int64_t rec = rec0 + kk;
#pragma unroll
    for (int side = 0; side < 2; ++side) {
        const uint8_t* bin = (const uint8_t*)(side ? a.V.sign : a.K.sign) + rec * kBinRecBytes;
        uint32_t* srow = reinterpret_cast<uint32_t*>(sb + (side ? Cfg::OFF_VSIGN : Cfg::OFF_KSIGN)) + kk * NWD;
#pragma unroll
        for (int w = 0; w < NWD; ++w) srow[w] = __ldg(reinterpret_cast<const uint32_t*>(bin) + w);
        reinterpret_cast<uint16_t*>(sb + (side ? Cfg::OFF_VBS : Cfg::OFF_KBS))[kk] =
            __ldg(reinterpret_cast<const unsigned short*>(bin + kBinScaleOff));
        if (COMP) {
            const uint16_t* res = reinterpret_cast<const uint16_t*>((const uint8_t*)(side ? a.V.nib : a.K.nib) +
                                                                    rec * kResRecBytes);
            uint8_t* nb = sb + (side ? Cfg::OFF_VNIB : Cfg::OFF_KNIB);
#pragma unroll
            for (int c = 0; c < NWD; ++c) {
                uint4 v;
                // two's-complement codes -> offset-binary (u = code + 8 per nibble)
                v.x = ((uint32_t)__ldg(res + 8 * c + 0) | ((uint32_t)__ldg(res + 8 * c + 1) << 16)) ^ 0x88888888u;
                v.y = ((uint32_t)__ldg(res + 8 * c + 2) | ((uint32_t)__ldg(res + 8 * c + 3) << 16)) ^ 0x88888888u;
                v.z = ((uint32_t)__ldg(res + 8 * c + 4) | ((uint32_t)__ldg(res + 8 * c + 5) << 16)) ^ 0x88888888u;
                v.w = ((uint32_t)__ldg(res + 8 * c + 6) | ((uint32_t)__ldg(res + 8 * c + 7) << 16)) ^ 0x88888888u;
                *reinterpret_cast<uint4*>(nb + nib_chunk_offset(kk, c, D)) = v;
            }
            reinterpret_cast<uint16_t*>(sb + (side ? Cfg::OFF_VRS : Cfg::OFF_KRS))[kk] = __ldg(res + 64);
        }
    }
}

template <int D, int GC, bool COMP>
__global__ void __launch_bounds__(kDecThreads) k_decode_records(const DecodeArgs a) {
    using Cfg = DecCfg<D, GC, COMP>;
    constexpr int T = Cfg::T;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = aligned_smem(smem_raw);
    const int warp = threadIdx.x >> 5;
    int slot, hg, split;
    cta_coords(a, slot, hg, split);
    const int s_begin = split * a.keys_per_split;
    const int s_end = min(a.seq_len, s_begin + a.keys_per_split);
    const int n_keys = max(0, s_end - s_begin);
    const int n_tiles = (n_keys + T - 1) / T;

    QState<D, GC> qs;
    prepare_query<D, GC, COMP, Cfg>(a, slot, hg, smem, qs);
    SoftState<GC, Cfg::NP> st;
    init_soft(st);
    const int64_t rec_base = (int64_t)slot * a.kv_stride + s_begin;
    for (int it = 0; it < n_tiles; ++it) {
        const int nk = min(T, n_keys - it * T);
        __syncthreads();
        load_tile_records<D, COMP, Cfg>(a, rec_base + it * T, nk, smem);
        __syncthreads();
        consume_warp_tile<D, GC, COMP, Cfg>(qs, st, smem, warp * 32, nk);
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

// Staging of a decode step's host-resident inputs (bc_stage_rows): every
// thread loads its 16-byte pieces of the segments (pinned host memory, over
// the host link) before waiting for the previous kernel in the stream, so the
// link latency overlaps that kernel's tail, then stores them to device memory.
// The decode kernel that follows (programmatic dependent launch) waits for
// this grid and reads its q rows from device memory: one host-link crossing
// per step instead of one per split CTA.
constexpr int kStageThreads = 256;
constexpr int kStageMaxSegs = 4;
constexpr int kStagePerThread = 4;  // 16-byte pieces a thread holds between the loads and the wait
struct StageArgs {
    const uint4* src[kStageMaxSegs];
    uint4* dst[kStageMaxSegs];
    int64_t n16[kStageMaxSegs];  // 16-byte pieces of each segment
    int n_segs;
};

__global__ void __launch_bounds__(kStageThreads) k_stage_rows(const StageArgs a) {
    uint4 v[kStagePerThread];
    int seg[kStagePerThread];
    int64_t idx[kStagePerThread];
    const int64_t first = ((int64_t)blockIdx.x * kStageThreads + threadIdx.x) * kStagePerThread;
#pragma unroll
    for (int j = 0; j < kStagePerThread; ++j) {
        int64_t i = first + j;
        seg[j] = -1;
        for (int s = 0; s < a.n_segs; ++s) {
            if (i < a.n16[s]) {
                seg[j] = s;
                idx[j] = i;
                v[j] = a.src[s][i];
                break;
            }
            i -= a.n16[s];
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
    for (int j = 0; j < kStagePerThread; ++j)
        if (seg[j] >= 0) a.dst[seg[j]][idx[j]] = v[j];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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


// Query heads handled per CTA, so that one read of every KV key serves them
// all: compensated caches at head dims 64 and 128 (tensor-core path) up to
// four heads of a slot's group, whose accumulators hold two heads per column
// tile; at 256 (tensor-core path, 64 accumulator registers per head pair) and
// at 32 (f32x2 value phase) two; binary caches BC_DEC_BIN_GC.
// The CTAs of a slot's remaining head groups, adjacent in the grid, share the
// KV tiles through L2.
int heads_per_cta(int group, int d, bool comp) {
    const int cap = comp ? ((BC_DEC_MMA && (d == 64 || d == 128)) ? BC_DEC_GQA_GC : 2) : BC_DEC_BIN_GC;
    return group < cap ? group : cap;
}

// Choose the split count so that all CTAs fit in one resident wave when the
// slots alone cannot fill the GPU (avoids a ragged second wave).
constexpr int kMaxKeysPerSplit = 32768 * kWarps;

Plan make_plan(int n_slots, int group, int seq_len, int d, bool comp, int capacity) {
    Plan p;
    p.gc = heads_per_cta(group, d, comp);
    p.n_hgroups = group / p.gc;
    p.tile = kTile;
    const int n_tiles = max(1, (seq_len + p.tile - 1) / p.tile);
    const int64_t units = (int64_t)n_slots * p.n_hgroups;
    int splits = 1;
    if (units < capacity) splits = (int)((int64_t)capacity * BC_DEC_WAVES / units);
    splits = max(1, min(splits, n_tiles / BC_DEC_MIN_TILES));
    if (BC_DEC_FILL && comp && units < capacity && splits < n_tiles) {
        // Compensated caches, where a CTA's split is long: when one wave
        // leaves many CTA slots idle, take the split count of up to four
        // waves whose last wave is fullest (C4: 278.6 against 297.5 us).
        // Binary CTAs are short, and extra waves cost them more than idle
        // slots (binary C4 105 against 97 us), so their plan stays one wave.
        auto fill = [&](int sp) {
            const int64_t ctas = units * sp;
            const int64_t waves = (ctas + capacity - 1) / capacity;
            return (double)ctas / (double)(waves * capacity);
        };
        if (fill(splits) < 0.93) {
            int best = splits;
            for (int sp = splits + 1; sp <= min(n_tiles, (int)(4 * (int64_t)capacity / units)); ++sp)
                if (fill(sp) > fill(best) + 0.02) best = sp;
            splits = best;
        }
    }
    // at most kMaxKeysPerSplit keys per CTA: the tensor-core value phase's
    // 32-bit accumulators take up to 32768 keys per warp
    splits = max(splits, (n_tiles * p.tile + kMaxKeysPerSplit - 1) / kMaxKeysPerSplit);
    const int tiles_per_split = (n_tiles + splits - 1) / splits;
    p.keys_per_split = tiles_per_split * p.tile;
    p.n_splits = max(1, (max(seq_len, 1) + p.keys_per_split - 1) / p.keys_per_split);
    return p;
}

// Workspace: ticket counters, then split partials (m, l, o[d]), then the
// entropy variant's split partials (m, z, w).
size_t ws_bytes_for(int n_slots, int group, int n_splits, int d, int n_hgroups) {
    const size_t part = (size_t)n_slots * group * n_splits * (d + 4) * sizeof(float);
    const size_t ent = (size_t)n_slots * group * n_splits * 3 * sizeof(float);
    const size_t cnt = (size_t)n_slots * n_hgroups * sizeof(unsigned);
    return ((part + 255) & ~(size_t)255) + ((cnt + 255) & ~(size_t)255) + ((ent + 255) & ~(size_t)255);
}

// Workspace bound over both modes: the counter region is sized for one head
// per CTA (the most counters), the partial region for the most splits.
size_t ws_bound(int n_slots, int group, int seq_len, int d) {
    size_t best = 0;
    for (int comp = 0; comp < 2; ++comp) {
        const Plan p = make_plan(n_slots, group, seq_len, d, comp != 0, kMaxCtasPlan);
        int splits = p.n_splits;
        if (BC_DEC_FILL && comp) {  // the fill search may pick up to four waves of splits at any capacity
            const int64_t units = (int64_t)n_slots * p.n_hgroups;
            const int n_tiles = max(1, (seq_len + p.tile - 1) / p.tile);
            if (units < kMaxCtasPlan) splits = max(splits, (int)std::min<int64_t>(n_tiles, 4 * (int64_t)kMaxCtasPlan / units));
        }
        const size_t b = ws_bytes_for(n_slots, group, splits, d, group);
        best = b > best ? b : best;
    }
    return best;
}

enum Variant { kVarPlanes = 0, kVarRecords = 1, kVarStep = 2, kVarEntropy = 3, kVarAdaptive = 4 };

template <int D, int GC, bool COMP>
int launch_decode(const DecodeArgs& a, int var, cudaStream_t st) {
    using Cfg = DecCfg<D, GC, COMP>;
    const unsigned grid = (unsigned)((int64_t)a.n_slots * a.n_hgroups * a.n_splits);
    if (grid == 0) return BC_OK;
    if constexpr (GC == 1) {
        if (var == kVarRecords) {
            k_decode_records<D, GC, COMP><<<grid, kDecThreads, Cfg::SMEM_B, st>>>(a);
            BC_LAUNCH_CHECK();
            return BC_OK;
        }
    }
    // Programmatic dependent launch: the CTAs of this kernel may be scheduled
    // while the previous kernel of the stream finishes (each waits in
    // griddepcontrol.wait before its first global access), which hides the
    // launch and ramp-up behind the previous kernel's tail.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = Cfg::SMEM_B;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaSuccess;
    if (var == kVarStep)
        e = cudaLaunchKernelEx(&cfg, k_decode_planes<D, GC, COMP, 1>, a);
    else if (var == kVarEntropy)
        e = cudaLaunchKernelEx(&cfg, k_decode_planes<D, GC, COMP, 2>, a);
    else if (var == kVarAdaptive) {
        if constexpr (COMP) e = cudaLaunchKernelEx(&cfg, k_decode_planes<D, GC, COMP, 3>, a);
    } else
        e = cudaLaunchKernelEx(&cfg, k_decode_planes<D, GC, COMP, 0>, a);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    BC_LAUNCH_CHECK();
    return BC_OK;
}

template <typename K>
int set_smem_and_occupancy(K kernel, int smem) {
    int per_sm = 1;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kDecThreads, smem);
    return per_sm;
}

// Sets the dynamic shared-memory limit of the kernel variant on the current
// device (once per device) and returns the resident-CTA capacity of the GPU.
template <int D, int GC, bool COMP>
int capacity_of(int var) {
    using Cfg = DecCfg<D, GC, COMP>;
    constexpr int kMaxDev = 64;
    static int cap[5][kMaxDev] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDev && cap[var][dev] > 0) return cap[var][dev];
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    bool done = false;
    if constexpr (GC == 1) {
        if (var == kVarRecords) {
            per_sm = set_smem_and_occupancy(k_decode_records<D, GC, COMP>, Cfg::SMEM_B);
            done = true;
        }
    }
    if constexpr (COMP) {
        if (var == kVarAdaptive) {
            per_sm = set_smem_and_occupancy(k_decode_planes<D, GC, COMP, 3>, Cfg::SMEM_B);
            done = true;
        }
    }
    if (!done)
        per_sm = (var == kVarStep)      ? set_smem_and_occupancy(k_decode_planes<D, GC, COMP, 1>, Cfg::SMEM_B)
                 : (var == kVarEntropy) ? set_smem_and_occupancy(k_decode_planes<D, GC, COMP, 2>, Cfg::SMEM_B)
                                        : set_smem_and_occupancy(k_decode_planes<D, GC, COMP, 0>, Cfg::SMEM_B);
    const int c = sms * max(1, per_sm);
    if (dev >= 0 && dev < kMaxDev) cap[var][dev] = c;
    return c;
}

// Adaptive caches: split the compensated segment (n_keep keys) and the
// binary one (seq_len - n_keep) so that one resident wave covers both, giving
// a binary split kBinKeysPerComp times the keys of a compensated split (a
// binary key costs about 40% of a compensated one).
#ifndef BC_DEC_BIN_HALVES
#define BC_DEC_BIN_HALVES 5
#endif
constexpr int kBinKeysPerComp = BC_DEC_BIN_HALVES;  // in halves: 2.5x
void plan_adaptive(DecodeArgs& a, int gc, int capacity) {
    const int n_hgroups = a.group / gc;
    const int64_t units = (int64_t)a.n_slots * n_hgroups;
    const int tiles_c = (a.n_keep + kTile - 1) / kTile;
    const int tiles_b = (a.seq_len - a.n_keep + kTile - 1) / kTile;
    const int eff = max(1, tiles_c + (tiles_b * 2 + kBinKeysPerComp - 1) / kBinKeysPerComp);
    int splits = units < capacity ? (int)(capacity / units) : 1;
    splits = max(1, min(splits, eff));
    const int tps = (eff + splits - 1) / splits;
    a.keys_per_split = tps * kTile;
    a.kps_bin = ((tps * kBinKeysPerComp + 1) / 2) * kTile;
    a.nc = (a.n_keep + a.keys_per_split - 1) / a.keys_per_split;
    const int nb = (a.seq_len - a.n_keep + a.kps_bin - 1) / a.kps_bin;
    a.n_splits = max(1, a.nc + nb);
    a.n_hgroups = n_hgroups;
}

// fit_ws: take fewer splits than planned when their partials would not fit
// in ws_bytes (the C++ launchers, whose scratch is a fixed array).
template <int D, int GC, bool COMP>
int run_decode_t(DecodeArgs a, int var, void* ws, size_t ws_bytes, cudaStream_t st, bool fit_ws) {
    const int cap = min(capacity_of<D, GC, COMP>(var), kMaxCtasPlan);
    if (var == kVarAdaptive) {
        plan_adaptive(a, GC, cap);
    } else {
        Plan p = make_plan(a.n_slots, a.group, a.seq_len, D, COMP, cap);
        a.n_splits = p.n_splits;
        a.keys_per_split = p.keys_per_split;
        a.n_hgroups = p.n_hgroups;
        if (fit_ws) {
            const int n_tiles = max(1, (a.seq_len + kTile - 1) / kTile);
            for (int sp = a.n_splits; a.n_splits > 1 && ws_bytes_for(a.n_slots, a.group, a.n_splits, D, a.n_hgroups) >
                                                          ws_bytes;) {
                sp = min(sp, a.n_splits) - 1;
                a.keys_per_split = ((n_tiles + sp - 1) / sp) * kTile;
                a.n_splits = max(1, (max(a.seq_len, 1) + a.keys_per_split - 1) / a.keys_per_split);
            }
            // the tensor-core value phase's accumulators bound the keys per CTA
            if (var != kVarRecords && DecCfg<D, GC, COMP>::MMA && a.keys_per_split > kMaxKeysPerSplit)
                return BC_ERR_TOO_LARGE;
        }
    }
    Plan p{a.n_splits, a.keys_per_split, a.n_hgroups, GC, kTile};
    if (p.n_splits > 1) {
        const size_t need = ws_bytes_for(a.n_slots, a.group, p.n_splits, D, p.n_hgroups);
        if (ws == nullptr || ws_bytes < need) return BC_ERR_WORKSPACE;
        // Ticket counters first, at a fixed offset: calls of any shape find them
        // zero (every completed call resets its own); partials follow and are
        // always written before they are read.
        const size_t cnt = (size_t)a.n_slots * p.n_hgroups * sizeof(unsigned);
        const size_t part = (size_t)a.n_slots * a.group * p.n_splits * (D + 4) * sizeof(float);
        uint8_t* base = reinterpret_cast<uint8_t*>(ws);
        a.ws_cnt = reinterpret_cast<unsigned*>(base);
        a.ws_part = reinterpret_cast<float*>(base + ((cnt + 255) & ~(size_t)255));
        a.ws_ent = reinterpret_cast<float*>(base + ((cnt + 255) & ~(size_t)255) + ((part + 255) & ~(size_t)255));
    } else {
        a.ws_part = nullptr;
        a.ws_cnt = nullptr;
        a.ws_ent = nullptr;
    }
    return launch_decode<D, GC, COMP>(a, var, st);
}

template <int D>
int run_decode_d(const DecodeArgs& a, bool comp, int var, void* ws, size_t wsb, cudaStream_t st, bool fit) {
    switch (heads_per_cta(a.group, D, comp)) {
        case 1:
            return comp ? run_decode_t<D, 1, true>(a, var, ws, wsb, st, fit)
                        : run_decode_t<D, 1, false>(a, var, ws, wsb, st, fit);
        case 2:
            return comp ? run_decode_t<D, 2, true>(a, var, ws, wsb, st, fit)
                        : run_decode_t<D, 2, false>(a, var, ws, wsb, st, fit);
        default:
            if constexpr (D == 64 || D == 128) {
                if (comp) return run_decode_t<D, 4, true>(a, var, ws, wsb, st, fit);
            }
            if (comp) return BC_ERR_UNSUPPORTED;
            return run_decode_t<D, 4, false>(a, var, ws, wsb, st, fit);
    }
}

int run_decode(const DecodeArgs& a, bool comp, int var, void* ws, size_t wsb, cudaStream_t st, bool fit = false) {
    switch (a.head_dim) {
        case 32: return run_decode_d<32>(a, comp, var, ws, wsb, st, fit);
        case 64: return run_decode_d<64>(a, comp, var, ws, wsb, st, fit);
        case 128: return run_decode_d<128>(a, comp, var, ws, wsb, st, fit);
        case 256: return run_decode_d<256>(a, comp, var, ws, wsb, st, fit);
        default: return BC_ERR_UNSUPPORTED;
    }
}

bool valid_group(int g) { return g == 1 || g == 2 || g == 4 || g == 8; }

// Default poll limit of an exchange word: 4096 fast polls, then 256 ns
// sleeps, about a second in all.
constexpr uint32_t kXchgSpinLimit = 1u << 22;

}  // namespace

namespace {

// Identity of the CUDA context current on this thread, unique for the life
// of the process (cuCtxGetCurrent and cuCtxGetId, reached through the
// runtime's driver entry points so the library does not link libcuda
// itself); 0 when no context is current or the entry points are missing.
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    });
    if (!get_current || !get_id) return 0;
    CUcontext c = nullptr;
    if (get_current(&c) != CUDA_SUCCESS || c == nullptr) return 0;
    unsigned long long id = 0;
    return get_id(c, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of a __device__ variable of this library on the current
// device.  In host code the variable's name is only a host-side stand-in, so
// the address is looked up with cudaGetSymbolAddress (with the device
// current) and cached per device together with the context it belongs to: a
// new context on the device (after cudaDeviceReset, say) reloads the module
// at another address, and the lookup is then made again.
struct SymbolAddressCache {
    static constexpr int kMaxDev = 64;
    std::mutex mu;
    void* addr[kMaxDev] = {};
    unsigned long long ctx[kMaxDev] = {};
};

int cached_symbol_address(SymbolAddressCache& c, const void* symbol, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    if (dev < 0 || dev >= SymbolAddressCache::kMaxDev) return BC_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(c.mu);
    const unsigned long long id = current_context_id();
    if (c.addr[dev] != nullptr && id != 0 && c.ctx[dev] == id) {
        *out = c.addr[dev];
        return BC_OK;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, symbol);  // also makes the device's primary context current
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    c.addr[dev] = p;
    c.ctx[dev] = current_context_id();
    *out = p;
    return BC_OK;
}

SymbolAddressCache g_error_word_addr;

}  // namespace

// Device address of the library's error word, for kernels compiled in other
// translation units (null when the lookup fails).
unsigned int* bc_device_error_ptr() {
    void* p = nullptr;
    return cached_symbol_address(g_error_word_addr, &g_bc_device_error, &p) == BC_OK ? static_cast<unsigned int*>(p)
                                                                                      : nullptr;
}

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
    return ws_bound(n_slots, group, seq_len, head_dim);
}

static int check_decode_args(const void* q, const bc_kv_planes& K, const bc_kv_planes& V, const void* out,
                             const float* partial, int n_slots, int group, int seq_len, int64_t kv_stride,
                             int head_dim, int mode) {
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
    return BC_OK;
}

static DecodeArgs decode_args(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial, int n_slots,
                              int group, int seq_len, int64_t kv_stride, int head_dim) {
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
    a.append_pos = -1;
    return a;
}

int bc_decode_attention(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial, int n_slots,
                        int group, int seq_len, int64_t kv_stride, int head_dim, int mode, void* workspace,
                        size_t workspace_bytes, void* stream) {
    const int rc = check_decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim, mode);
    if (rc != BC_OK || n_slots == 0) return rc;
    const DecodeArgs a = decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim);
    return run_decode(a, mode == BC_MODE_COMPENSATED, kVarPlanes, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t bc_xchg_bytes(int n_heads, int head_dim, int world) {
    if (n_heads <= 0 || world <= 0 || world > 8 || !bc_valid_head_dim(head_dim)) return 0;
    const size_t words = (size_t)2 * world * n_heads * (head_dim + 2) * sizeof(unsigned long long);
    return (words + 255) & ~(size_t)255;
}

int bc_xchg_alloc(size_t bytes, void** buf) {
    if (!buf || bytes == 0) return BC_ERR_ARG;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return BC_ERR_CUDA_BASE + (int)e;
    }
    *buf = p;
    return BC_OK;
}

int bc_xchg_free(void* buf) {
    const cudaError_t e = cudaFree(buf);
    return e == cudaSuccess ? BC_OK : BC_ERR_CUDA_BASE + (int)e;
}

int bc_ipc_handle(const void* buf, void* handle) {
    if (!buf || !handle) return BC_ERR_ARG;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(buf));
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
    memcpy(handle, &h, sizeof(h));
    return BC_OK;
}

int bc_ipc_open(const void* handle, void** buf) {
    if (!handle || !buf) return BC_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? BC_OK : BC_ERR_CUDA_BASE + (int)e;
}

int bc_ipc_close(void* buf) {
    const cudaError_t e = cudaIpcCloseMemHandle(buf);
    return e == cudaSuccess ? BC_OK : BC_ERR_CUDA_BASE + (int)e;
}

int bc_decode_attention_xchg(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, int n_slots, int group,
                             int seq_len, int64_t kv_stride, int head_dim, int mode, bc_xchg x, void* workspace,
                             size_t workspace_bytes, void* stream) {
    const int rc = check_decode_args(q, K, V, out, nullptr, n_slots, group, seq_len, kv_stride, head_dim, mode);
    if (rc != BC_OK || n_slots == 0) return rc;
    if (!out || x.world < 1 || x.world > 8 || x.rank < 0 || x.rank >= x.world || x.epoch == 0) return BC_ERR_ARG;
    // Every rank's buffer must hold both parity halves of this call's triples:
    // the kernel stores into all of them and reads its own.
    const uint64_t need = (uint64_t)2 * x.world * ((uint64_t)n_slots * group) * (head_dim + 2) * 8;
    if (x.buf_bytes < need) return BC_ERR_ARG;
    DecodeArgs a = decode_args(q, K, V, out, nullptr, n_slots, group, seq_len, kv_stride, head_dim);
    for (int j = 0; j < x.world; ++j) {
        if (!x.bufs[j] || !bc_aligned(x.bufs[j], 256)) return BC_ERR_ARG;
        a.xparts[j] = reinterpret_cast<unsigned long long*>(x.bufs[j]);
    }
    a.xw = x.world;
    a.xrank = x.rank;
    a.xepoch = x.epoch;
    a.xspin = x.spin_limit ? x.spin_limit : kXchgSpinLimit;
    return run_decode(a, mode == BC_MODE_COMPENSATED, kVarPlanes, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t bc_decode_adaptive_workspace_bytes(int n_slots, int group, int seq_len, int n_keep, int head_dim) {
    if (n_slots <= 0 || !valid_group(group) || seq_len < 0 || n_keep < 0 || n_keep > seq_len ||
        !bc_valid_head_dim(head_dim))
        return 0;
    size_t best = 0;
    for (int gc = 1; gc <= 4 && gc <= group; gc *= 2) {  // compensated CTAs hold one, two or four heads
        DecodeArgs a{};
        a.n_slots = n_slots;
        a.group = group;
        a.seq_len = seq_len;
        a.n_keep = n_keep;
        plan_adaptive(a, gc, kMaxCtasPlan);
        const size_t b = ws_bytes_for(n_slots, group, a.n_splits, head_dim, group);
        best = b > best ? b : best;
    }
    return best;
}

int bc_decode_attention_adaptive(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial,
                                 int n_slots, int group, int seq_len, int n_keep, int64_t kv_stride,
                                 int64_t res_stride, int head_dim, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    const int rc = check_decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim,
                                     BC_MODE_COMPENSATED);
    if (rc != BC_OK || n_slots == 0) return rc;
    const int b0 = (n_keep + 7) & ~7;
    if (n_keep < 0 || n_keep > seq_len || kv_stride < (int64_t)b0 + (seq_len - n_keep) || res_stride < n_keep)
        return BC_ERR_ARG;
    if (res_stride % 8 != 0) return BC_ERR_ALIGN;
    DecodeArgs a = decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim);
    a.n_keep = n_keep;
    a.b0 = b0;
    a.res_stride = res_stride;
    return run_decode(a, true, kVarAdaptive, workspace, workspace_bytes, (cudaStream_t)stream);
}

int bc_decode_attention_entropy(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial,
                                float* entropy, int n_slots, int group, int seq_len, int64_t kv_stride, int head_dim,
                                int mode, void* workspace, size_t workspace_bytes, void* stream) {
    const int rc = check_decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim, mode);
    if (rc != BC_OK || n_slots == 0) return rc;
    if (!entropy) return BC_ERR_ARG;
    if (!bc_aligned(entropy, 4)) return BC_ERR_ALIGN;
    DecodeArgs a = decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim);
    a.entropy = entropy;
    return run_decode(a, mode == BC_MODE_COMPENSATED, kVarEntropy, workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"

namespace {
// Where the fused step's host-side operands live: bit 0 q, bit 1 new_k and
// new_v in pinned (page-locked) host memory, which kernels read through
// unified addressing; -1 for pageable host memory, which they cannot.
int host_inputs(const void* q, const void* new_k, const void* new_v, const void* out) {
    auto kind = [](const void* p) -> int {  // 0 device / managed / null, 1 pinned host, -1 pageable
        if (!p) return 0;
        cudaPointerAttributes at;
        if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        if (at.type == cudaMemoryTypeHost) return 1;
        return at.type == cudaMemoryTypeUnregistered ? -1 : 0;
    };
    const int kq = kind(q), kk = kind(new_k), kv = kind(new_v), ko = kind(out);
    if (kq < 0 || kk < 0 || kv < 0 || ko < 0) return -1;
    // The new rows are read early only when both are host-resident: a device
    // row may still be written by the kernel queued ahead of this one.
    return (kq ? 1 : 0) | ((kk && kv) ? 2 : 0);
}
}  // namespace

extern "C" {

int bc_decode_step(const void* q, const void* new_k, const void* new_v, bc_kv_planes K, bc_kv_planes V, void* out,
                   float* partial, int n_slots, int group, int seq_len, int64_t kv_stride, int head_dim, int mode,
                   int append_pos, int append_res, void* workspace, size_t workspace_bytes, void* stream) {
    const int rc = check_decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim, mode);
    if (rc != BC_OK || n_slots == 0) return rc;
    if (append_pos < -1 || append_pos >= seq_len) return BC_ERR_ARG;
    DecodeArgs a = decode_args(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim);
    if (append_pos >= 0) {
        if (append_res != BC_RES_NONE && append_res != BC_RES_FP16_SCALE && append_res != BC_RES_FP32_SCALE)
            return BC_ERR_ARG;
        // compensated attention reads the residual of the appended row
        if (mode == BC_MODE_COMPENSATED && append_res == BC_RES_NONE) return BC_ERR_ARG;
        if (!new_k || !new_v) return BC_ERR_ARG;
        if (append_res != BC_RES_NONE && (!K.nib || !K.rscale || !V.nib || !V.rscale)) return BC_ERR_ARG;
        if (append_res != BC_RES_NONE && (!bc_aligned(K.nib, 16) || !bc_aligned(V.nib, 16))) return BC_ERR_ALIGN;
        if (!bc_aligned(new_k, 2) || !bc_aligned(new_v, 2)) return BC_ERR_ALIGN;
        a.new_k = (const __half*)new_k;
        a.new_v = (const __half*)new_v;
        a.append_pos = append_pos;
        a.append_res = append_res;
    }
    const int hi = host_inputs(q, a.new_k, a.new_v, out);
    if (hi < 0) return BC_ERR_ARG;
    a.host_in = hi;
    return run_decode(a, mode == BC_MODE_COMPENSATED, kVarStep, workspace, workspace_bytes, (cudaStream_t)stream);
}

int bc_decode_step_paged(const void* q, const void* new_k, const void* new_v, bc_kv_planes K, bc_kv_planes V,
                         void* out, float* partial, bc_page_table pt, int n_slots, int group, int seq_len,
                         int head_dim, int mode, int append_pos, int append_res, void* workspace,
                         size_t workspace_bytes, void* stream) {
    if (!pt.pages || pt.page_size <= 0 || pt.page_size % kTile != 0 || pt.n_pages <= 0 || pt.max_pages <= 0)
        return BC_ERR_ARG;
    if ((int64_t)pt.max_pages * pt.page_size < seq_len) return BC_ERR_ARG;
    if (!bc_aligned(pt.pages, 4)) return BC_ERR_ALIGN;
    // the pool is checked as a contiguous cache of n_pages slots of page_size positions
    const int rc = check_decode_args(q, K, V, out, partial, n_slots, group, 0, pt.page_size, head_dim, mode);
    if (rc != BC_OK || n_slots == 0) return rc;
    if (seq_len < 0 || append_pos < -1 || append_pos >= seq_len) return BC_ERR_ARG;
    DecodeArgs a = decode_args(q, K, V, out, partial, n_slots, group, seq_len, pt.page_size, head_dim);
    a.pages = pt.pages;
    a.max_pages = pt.max_pages;
    a.page_size = pt.page_size;
    a.n_pages = pt.n_pages;
    if (append_pos >= 0) {
        if (append_res != BC_RES_NONE && append_res != BC_RES_FP16_SCALE && append_res != BC_RES_FP32_SCALE)
            return BC_ERR_ARG;
        if (mode == BC_MODE_COMPENSATED && append_res == BC_RES_NONE) return BC_ERR_ARG;
        if (!new_k || !new_v) return BC_ERR_ARG;
        if (append_res != BC_RES_NONE && (!K.nib || !K.rscale || !V.nib || !V.rscale)) return BC_ERR_ARG;
        if (append_res != BC_RES_NONE && (!bc_aligned(K.nib, 16) || !bc_aligned(V.nib, 16))) return BC_ERR_ALIGN;
        if (!bc_aligned(new_k, 2) || !bc_aligned(new_v, 2)) return BC_ERR_ALIGN;
        a.new_k = (const __half*)new_k;
        a.new_v = (const __half*)new_v;
        a.append_pos = append_pos;
        a.append_res = append_res;
    }
    const int hi = host_inputs(q, a.new_k, a.new_v, out);
    if (hi < 0) return BC_ERR_ARG;
    a.host_in = hi;
    return run_decode(a, mode == BC_MODE_COMPENSATED, kVarStep, workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"

// Scratch of the C++ record launchers (launch_binary_attention,
// launch_compensated_attention).  The reference's launchers take no workspace
// and allocate nothing (compensated_attention.cu:111-134), so their
// replacements keep the split-K partials in a fixed array of the library
// (every GPU that loads the library holds it until exit) and plan fewer
// splits for shapes whose partials would not fit.
namespace {
constexpr size_t kLauncherScratchBytes = size_t(4) << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_bc_launcher_scratch[kLauncherScratchBytes];
SymbolAddressCache g_launcher_scratch_addr;
}  // namespace

extern "C" {

size_t bc_attention_workspace_bytes(int batch, int n_heads, int seq_len, int head_dim) {
    if (batch <= 0 || n_heads <= 0) return 0;
    return bc_decode_workspace_bytes(batch * n_heads, 1, seq_len, head_dim);
}

static int record_attention(const void* q, const void* kb, const void* kr, const void* vb, const void* vr, void* out,
                            int batch, int n_heads, int seq_len, int head_dim, bool comp, void* ws, size_t wsb,
                            void* stream, bool fixed_scratch = false) {
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
    if (fixed_scratch) {
        const int rc = cached_symbol_address(g_launcher_scratch_addr, g_bc_launcher_scratch, &ws);
        if (rc != BC_OK) return rc;
        wsb = kLauncherScratchBytes;
        // The ticket counters (one per head: one head per CTA here) must start
        // at zero; the array keeps whatever the previous call left there.
        const cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)n * sizeof(unsigned), (cudaStream_t)stream);
        if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    }
    return run_decode(a, comp, kVarRecords, ws, wsb, (cudaStream_t)stream, fixed_scratch);
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

int bc_stage_rows(const bc_copy_seg* segs, int n_segs, void* stream) {
    if (n_segs < 0 || n_segs > kStageMaxSegs || (n_segs > 0 && !segs)) return BC_ERR_ARG;
    StageArgs a{};
    int64_t total = 0;
    a.n_segs = n_segs;
    for (int s = 0; s < n_segs; ++s) {
        if (segs[s].bytes % 16 != 0) return BC_ERR_ALIGN;
        if (segs[s].bytes > 0 && (!segs[s].src || !segs[s].dst)) return BC_ERR_ARG;
        if (!bc_aligned(segs[s].src, 16) || !bc_aligned(segs[s].dst, 16)) return BC_ERR_ALIGN;
        a.src[s] = reinterpret_cast<const uint4*>(segs[s].src);
        a.dst[s] = reinterpret_cast<uint4*>(segs[s].dst);
        a.n16[s] = (int64_t)(segs[s].bytes / 16);
        total += a.n16[s];
    }
    if (total == 0) return BC_OK;
    const int64_t per_cta = (int64_t)kStageThreads * kStagePerThread;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((total + per_cta - 1) / per_cta));
    cfg.blockDim = dim3(kStageThreads);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_stage_rows, a);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    BC_LAUNCH_CHECK();
    return BC_OK;
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

int bc_record_attention_fixed_scratch(const void* q, const void* k_bin, const void* k_res, const void* v_bin,
                                      const void* v_res, void* out, int batch, int n_heads, int seq_len, int head_dim,
                                      bool compensated, void* stream) {
    return record_attention(q, k_bin, k_res, v_bin, v_res, out, batch, n_heads, seq_len, head_dim, compensated,
                            nullptr, 0, stream, true);
}

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

SymbolAddressCache g_static_scratch_addr;

// Device address of the array on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up
// (with the device current) on the first call on each device and cached;
// the lookup is made again when the device has a new context.
int static_scratch_address(void** addr) {
    return cached_symbol_address(g_static_scratch_addr, g_bc_static_scratch, addr);
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
    const size_t counter_bytes = (size_t)n_slots * group * sizeof(unsigned);  // counters of any mode
    cudaError_t e = cudaMemsetAsync(scratch, 0, counter_bytes, (cudaStream_t)stream);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    return bc_decode_attention(q, K, V, out, partial, n_slots, group, seq_len, kv_stride, head_dim, mode, scratch,
                               kStaticScratchBytes, stream);
}

}  // extern "C"
