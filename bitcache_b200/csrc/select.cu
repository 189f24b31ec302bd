// Per-vector adaptive precision: keep the INT4 residual only for the n_keep
// vectors of each slot with the largest residual energy, store the rest
// binary-only.  sm_100a.
//
// There is no reference kernel for this (the reference's adaptive precision
// is per head, adaptive_precision.cu).  The selection key of a vector is
//     key = fp32(rs * rs) * (float)sum_i code_i^2        (rs = fp16 residual scale)
// a non-negative float, so its bit pattern orders like an unsigned integer.
// Ties go to the lower position.  One CTA per slot:
//   1. keys of the slot's seq_len vectors into the workspace;
//   2. MSB-first radix select (4 passes of 8 bits) for the n_keep-th largest
//      key K* and the count of keys above it;
//   3. an ordered block scan over positions keeps the first
//      (n_keep - count_above) keys equal to K*.
// With apply != 0 the unselected vectors' residual scale is set to 0 and
// their codes to 0, so they contribute exactly nothing in compensated
// attention.
#include "common.cuh"

namespace bc {

constexpr int kSelThreads = 256;

template <int D>
__device__ __forceinline__ uint32_t residual_key(const uint8_t* nib, const __half* rscale, int64_t row) {
    int ss = 0;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
        const uint4 ch = *reinterpret_cast<const uint4*>(nib + nib_chunk_offset(row, c, D));
        const uint32_t w[4] = {ch.x, ch.y, ch.z, ch.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int n = (int)((w[k] >> (4 * j)) & 0xFu) - 8;  // offset-binary
                ss += n * n;
            }
    }
    const float rs = __half2float(rscale[row]);
    const float rr = rs * rs;
    return __float_as_uint(rr * (float)ss);
}

// JOINT: one choice per position for the K and V planes together, keyed by
// the fp32 sum of the two vectors' keys (P2 = the V planes).
template <int D, bool JOINT>
__global__ void __launch_bounds__(kSelThreads) k_select_topk(bc_kv_planes P, bc_kv_planes P2, int seq_len,
                                                             int64_t kv_stride, int n_keep,
                                                             uint32_t* __restrict__ keys,
                                                             uint8_t* __restrict__ keep, int apply) {
    const int slot = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t base = (int64_t)slot * kv_stride;
    uint32_t* skeys = keys + base;
    const uint8_t* nib = reinterpret_cast<const uint8_t*>(P.nib);
    const __half* rsc = reinterpret_cast<const __half*>(P.rscale);
    for (int s = tid; s < seq_len; s += kSelThreads) {
        uint32_t key = residual_key<D>(nib, rsc, base + s);
        if (JOINT)
            key = __float_as_uint(__uint_as_float(key) + __uint_as_float(residual_key<D>(
                                      reinterpret_cast<const uint8_t*>(P2.nib),
                                      reinterpret_cast<const __half*>(P2.rscale), base + s)));
        skeys[s] = key;
    }
    __syncthreads();

    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_k, s_above;
    __shared__ uint32_t warp_sums[kSelThreads / 32];
    uint32_t prefix = 0, mask = 0;
    uint32_t k = (uint32_t)min(max(n_keep, 0), seq_len);  // rank (1-based) of K* among the largest
    uint32_t above = 0;                                   // keys strictly greater than the prefix range
    const bool select_all = n_keep >= seq_len, select_none = n_keep <= 0;
    if (!select_all && !select_none) {
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
            __syncthreads();
            for (int s = tid; s < seq_len; s += kSelThreads) {
                const uint32_t key = skeys[s];
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                // walk digits from the largest down until the k-th largest is reached
                uint32_t cum = 0;
                int dsel = 0;
                for (int dgt = 255; dgt >= 0; --dgt) {
                    if (cum + hist[dgt] >= k) {
                        dsel = dgt;
                        break;
                    }
                    cum += hist[dgt];
                }
                s_prefix = prefix | ((uint32_t)dsel << shift);
                s_k = k - cum;
                s_above = above + cum;
            }
            __syncthreads();
            prefix = s_prefix;
            k = s_k;
            above = s_above;
            mask |= 0xFFu << shift;
            __syncthreads();
        }
    }
    // K* = prefix; `above` keys are greater; keep the first k keys equal to K*.
    const uint32_t kstar = prefix;
    uint32_t taken = 0;  // ties kept so far (uniform)
    const int lane = tid & 31, warp = tid >> 5;
    for (int s0 = 0; s0 < seq_len; s0 += kSelThreads) {
        const int s = s0 + tid;
        const bool in = s < seq_len;
        const uint32_t key = in ? skeys[s] : 0u;
        const bool tie = in && !select_all && !select_none && key == kstar;
        const uint32_t ballot = __ballot_sync(0xffffffffu, tie);
        if (lane == 0) warp_sums[warp] = __popc(ballot);
        __syncthreads();
        uint32_t before = 0, total = 0;
        for (int w = 0; w < kSelThreads / 32; ++w) {
            if (w < warp) before += warp_sums[w];
            total += warp_sums[w];
        }
        before += __popc(ballot & ((1u << lane) - 1u));
        if (in) {
            bool kept;
            if (select_all) kept = true;
            else if (select_none) kept = false;
            else kept = key > kstar || (tie && taken + before < k);
            if (keep) keep[base + s] = kept ? 1 : 0;
            if (apply && !kept) {
                reinterpret_cast<uint16_t*>(P.rscale)[base + s] = 0;
                uint8_t* nb = reinterpret_cast<uint8_t*>(P.nib);
#pragma unroll
                for (int c = 0; c < D / 32; ++c)
                    *reinterpret_cast<uint4*>(nb + nib_chunk_offset(base + s, c, D)) =
                        make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // codes 0
            }
        }
        taken += total;
        __syncthreads();
    }
    (void)above;
}

// Stable partition of each slot's positions into the compact adaptive layout:
// kept positions (keep != 0) move to rows [0, n_keep) of the sign/scale planes
// and of the residual planes (row stride r_stride); the others, binary only,
// to rows [b0, b0 + seq_len - n_keep) of the sign/scale planes, b0 = n_keep
// rounded up to 8.  K and V move together (keep is per position).  One CTA
// per slot; a block scan over the keep mask gives each position's new row.
template <int D>
__global__ void __launch_bounds__(kSelThreads) k_compact_adaptive(bc_kv_planes K, bc_kv_planes V,
                                                                  const uint8_t* __restrict__ keep, int seq_len,
                                                                  int64_t kv_stride, bc_kv_planes Kc,
                                                                  bc_kv_planes Vc, int64_t c_stride,
                                                                  int64_t r_stride, int b0) {
    constexpr int NWD = D / 32;
    const int slot = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ uint32_t warp_sums[kSelThreads / 32];
    int kept_before = 0;  // kept positions in earlier chunks (uniform)
    for (int s0 = 0; s0 < seq_len; s0 += kSelThreads) {
        const int s = s0 + tid;
        const bool in = s < seq_len;
        const bool kp = in && keep[(int64_t)slot * kv_stride + s] != 0;
        const uint32_t ballot = __ballot_sync(0xffffffffu, kp);
        if (lane == 0) warp_sums[warp] = __popc(ballot);
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < kSelThreads / 32; ++w) {
            if (w < warp) before += (int)warp_sums[w];
            total += (int)warp_sums[w];
        }
        before += __popc(ballot & ((1u << lane) - 1u));
        if (in) {
            const int rank = kept_before + before;  // kept positions before s
            const int64_t src = (int64_t)slot * kv_stride + s;
            const int64_t dst = (int64_t)slot * c_stride + (kp ? rank : b0 + (s - rank));
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const bc_kv_planes& A = j ? V : K;
                const bc_kv_planes& C = j ? Vc : Kc;
                const uint32_t* ss = reinterpret_cast<const uint32_t*>(A.sign) + src * NWD;
                uint32_t* ds = reinterpret_cast<uint32_t*>(C.sign) + dst * NWD;
#pragma unroll
                for (int k = 0; k < NWD; ++k) ds[k] = ss[k];
                reinterpret_cast<uint16_t*>(C.bscale)[dst] = reinterpret_cast<const uint16_t*>(A.bscale)[src];
                if (kp) {
                    const int64_t rdst = (int64_t)slot * r_stride + rank;
#pragma unroll
                    for (int c = 0; c < NWD; ++c)
                        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(C.nib) + nib_chunk_offset(rdst, c, D)) =
                            *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(A.nib) +
                                                            nib_chunk_offset(src, c, D));
                    reinterpret_cast<uint16_t*>(C.rscale)[rdst] = reinterpret_cast<const uint16_t*>(A.rscale)[src];
                }
            }
        }
        kept_before += total;
        __syncthreads();
    }
}

}  // namespace bc

using namespace bc;

extern "C" {

size_t bc_select_workspace_bytes(int n_slots, int64_t kv_stride) {
    if (n_slots <= 0 || kv_stride <= 0) return 0;
    return (size_t)n_slots * (size_t)kv_stride * sizeof(uint32_t);
}

int bc_select_residual_topk(bc_kv_planes P, int n_slots, int seq_len, int64_t kv_stride, int head_dim, int n_keep,
                            uint8_t* keep, int apply, void* workspace, size_t workspace_bytes, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) return BC_ERR_UNSUPPORTED;
    if (n_slots < 0 || seq_len < 0 || kv_stride < seq_len) return BC_ERR_ARG;
    if (n_slots == 0 || seq_len == 0) return BC_OK;
    if (!P.nib || !P.rscale || (!keep && !apply)) return BC_ERR_ARG;
    if (kv_stride % 8 != 0 || !bc_aligned(P.nib, 16)) return BC_ERR_ALIGN;
    if (!workspace || workspace_bytes < bc_select_workspace_bytes(n_slots, kv_stride)) return BC_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    uint32_t* keys = reinterpret_cast<uint32_t*>(workspace);
    const bc_kv_planes none{};
    switch (head_dim) {
        case 32: k_select_topk<32, false><<<n_slots, kSelThreads, 0, st>>>(P, none, seq_len, kv_stride, n_keep, keys, keep, apply); break;
        case 64: k_select_topk<64, false><<<n_slots, kSelThreads, 0, st>>>(P, none, seq_len, kv_stride, n_keep, keys, keep, apply); break;
        case 128: k_select_topk<128, false><<<n_slots, kSelThreads, 0, st>>>(P, none, seq_len, kv_stride, n_keep, keys, keep, apply); break;
        default: k_select_topk<256, false><<<n_slots, kSelThreads, 0, st>>>(P, none, seq_len, kv_stride, n_keep, keys, keep, apply); break;
    }
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_select_positions_topk(bc_kv_planes K, bc_kv_planes V, int n_slots, int seq_len, int64_t kv_stride,
                             int head_dim, int n_keep, uint8_t* keep, void* workspace, size_t workspace_bytes,
                             void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) return BC_ERR_UNSUPPORTED;
    if (n_slots < 0 || seq_len < 0 || kv_stride < seq_len) return BC_ERR_ARG;
    if (n_slots == 0 || seq_len == 0) return BC_OK;
    if (!K.nib || !K.rscale || !V.nib || !V.rscale || !keep) return BC_ERR_ARG;
    if (kv_stride % 8 != 0 || !bc_aligned(K.nib, 16) || !bc_aligned(V.nib, 16)) return BC_ERR_ALIGN;
    if (!workspace || workspace_bytes < bc_select_workspace_bytes(n_slots, kv_stride)) return BC_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    uint32_t* keys = reinterpret_cast<uint32_t*>(workspace);
    switch (head_dim) {
        case 32: k_select_topk<32, true><<<n_slots, kSelThreads, 0, st>>>(K, V, seq_len, kv_stride, n_keep, keys, keep, 0); break;
        case 64: k_select_topk<64, true><<<n_slots, kSelThreads, 0, st>>>(K, V, seq_len, kv_stride, n_keep, keys, keep, 0); break;
        case 128: k_select_topk<128, true><<<n_slots, kSelThreads, 0, st>>>(K, V, seq_len, kv_stride, n_keep, keys, keep, 0); break;
        default: k_select_topk<256, true><<<n_slots, kSelThreads, 0, st>>>(K, V, seq_len, kv_stride, n_keep, keys, keep, 0); break;
    }
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_compact_adaptive(bc_kv_planes K, bc_kv_planes V, const uint8_t* keep, int n_slots, int seq_len,
                        int64_t kv_stride, int head_dim, int n_keep, bc_kv_planes Kc, bc_kv_planes Vc,
                        int64_t c_stride, int64_t r_stride, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) return BC_ERR_UNSUPPORTED;
    if (n_slots < 0 || seq_len < 0 || kv_stride < seq_len || n_keep < 0 || n_keep > seq_len) return BC_ERR_ARG;
    const int b0 = (n_keep + 7) & ~7;
    if (c_stride < (int64_t)b0 + (seq_len - n_keep) || r_stride < b0) return BC_ERR_ARG;
    if (n_slots == 0 || seq_len == 0) return BC_OK;
    const bc_kv_planes* all[4] = {&K, &V, &Kc, &Vc};
    for (const bc_kv_planes* P : all) {
        if (!P->sign || !P->bscale || !P->nib || !P->rscale) return BC_ERR_ARG;
        if (!bc_aligned(P->nib, 16) || !bc_aligned(P->sign, 16)) return BC_ERR_ALIGN;
    }
    if (!keep) return BC_ERR_ARG;
    if (kv_stride % 8 != 0 || c_stride % 8 != 0 || r_stride % 8 != 0) return BC_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    switch (head_dim) {
        case 32: k_compact_adaptive<32><<<n_slots, kSelThreads, 0, st>>>(K, V, keep, seq_len, kv_stride, Kc, Vc, c_stride, r_stride, b0); break;
        case 64: k_compact_adaptive<64><<<n_slots, kSelThreads, 0, st>>>(K, V, keep, seq_len, kv_stride, Kc, Vc, c_stride, r_stride, b0); break;
        case 128: k_compact_adaptive<128><<<n_slots, kSelThreads, 0, st>>>(K, V, keep, seq_len, kv_stride, Kc, Vc, c_stride, r_stride, b0); break;
        default: k_compact_adaptive<256><<<n_slots, kSelThreads, 0, st>>>(K, V, keep, seq_len, kv_stride, Kc, Vc, c_stride, r_stride, b0); break;
    }
    BC_LAUNCH_CHECK();
    return BC_OK;
}

}  // extern "C"
