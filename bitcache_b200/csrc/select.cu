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

template <int D>
__global__ void __launch_bounds__(kSelThreads) k_select_topk(bc_kv_planes P, int seq_len, int64_t kv_stride,
                                                             int n_keep, uint32_t* __restrict__ keys,
                                                             uint8_t* __restrict__ keep, int apply) {
    const int slot = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t base = (int64_t)slot * kv_stride;
    uint32_t* skeys = keys + base;
    const uint8_t* nib = reinterpret_cast<const uint8_t*>(P.nib);
    const __half* rsc = reinterpret_cast<const __half*>(P.rscale);
    for (int s = tid; s < seq_len; s += kSelThreads) skeys[s] = residual_key<D>(nib, rsc, base + s);
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
    switch (head_dim) {
        case 32: k_select_topk<32><<<n_slots, kSelThreads, 0, st>>>(P, seq_len, kv_stride, n_keep, keys, keep, apply); break;
        case 64: k_select_topk<64><<<n_slots, kSelThreads, 0, st>>>(P, seq_len, kv_stride, n_keep, keys, keep, apply); break;
        case 128: k_select_topk<128><<<n_slots, kSelThreads, 0, st>>>(P, seq_len, kv_stride, n_keep, keys, keep, apply); break;
        default: k_select_topk<256><<<n_slots, kSelThreads, 0, st>>>(P, seq_len, kv_stride, n_keep, keys, keep, apply); break;
    }
    BC_LAUNCH_CHECK();
    return BC_OK;
}

}  // extern "C"
