// Attention entropy over binary scores and precision selection (reference
// adaptive_precision.cu), sm_100a.
//
// compute_head_entropy_kernel (adaptive_precision.cu:13-130) walks every key
// twice (max, then sum of exp and exp*score) with one 128-thread block per
// head.  Here one 256-thread CTA per head makes a single pass: each thread
// keeps an online (max, sum exp, sum exp*score) triple over its keys and the
// triples are merged with the log-sum-exp rule, giving
//   H = log Z + max - W / max(Z, 1e-12),  Z = sum e^(s-max), W = sum e^(s-max) s.
// Scores carry no 1/sqrt(d) factor, as in the reference (:74-75); the query
// scale uses the reference's 128-thread tree order (:46-59).
#include "common.cuh"

namespace bc {

constexpr int kEntThreads = 256;

struct EntState {
    float m, z, w;
};

__device__ __forceinline__ EntState ent_merge(EntState a, EntState b) {
    const float M = fmaxf(a.m, b.m);
    if (M == -INFINITY) return a;
    const float fa = (a.m == -INFINITY) ? 0.0f : __expf(a.m - M);
    const float fb = (b.m == -INFINITY) ? 0.0f : __expf(b.m - M);
    return EntState{M, a.z * fa + b.z * fb, a.w * fa + b.w * fb};
}

// records != 0: k_sign is a BinaryVec array ([n_heads][seq_len], kv_stride = seq_len);
// otherwise a sign plane with the scale plane in k_scale.
template <int NW, bool RECORDS>
__global__ void __launch_bounds__(kEntThreads) k_head_entropy(const __half* __restrict__ q,
                                                              const uint8_t* __restrict__ k_sign,
                                                              const __half* __restrict__ k_scale,
                                                              float* __restrict__ out, int seq_len,
                                                              int64_t kv_stride, int head_dim) {
    const int h = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ uint32_t s_qsign[8];
    __shared__ float s_scale;
    __shared__ EntState s_part[kEntThreads / 32];
    if (warp == 0) {
        float x[NW];
#pragma unroll
        for (int k = 0; k < NW; ++k) x[k] = __half2float(q[(int64_t)h * head_dim + 32 * k + lane]);
#pragma unroll
        for (int k = 0; k < NW; ++k) {
            const uint32_t w = __ballot_sync(0xffffffffu, x[k] >= 0.0f);
            if (lane == 0) s_qsign[k] = w;
        }
        // 128-thread tree order of the reference block reduction
        float p7[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float s = 0.0f;
            if (k < NW) s += fabsf(x[k]);
            if (k + 4 < NW) s += fabsf(x[k + 4]);
            p7[k] = s;
        }
        float v = (p7[0] + p7[2]) + (p7[1] + p7[3]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) s_scale = v / (float)head_dim;
    }
    __syncthreads();
    uint32_t qs[NW];
#pragma unroll
    for (int k = 0; k < NW; ++k) qs[k] = s_qsign[k];
    const float scale_q = s_scale;
    EntState st{-INFINITY, 0.0f, 0.0f};
    const int64_t base = (int64_t)h * kv_stride;
    for (int s = tid; s < seq_len; s += kEntThreads) {
        const int64_t idx = base + s;
        int pop = 0;
        float ks;
        if (RECORDS) {
            const uint8_t* rec = k_sign + idx * kBinRecBytes;
#pragma unroll
            for (int k = 0; k < NW; ++k) pop += __popc(~(qs[k] ^ __ldg(reinterpret_cast<const uint32_t*>(rec) + k)));
            ks = __half2float(__ldg(reinterpret_cast<const __half*>(rec + kBinScaleOff)));
        } else {
            const uint32_t* row = reinterpret_cast<const uint32_t*>(k_sign) + idx * NW;
#pragma unroll
            for (int k = 0; k < NW; ++k) pop += __popc(~(qs[k] ^ __ldg(row + k)));
            ks = __half2float(k_scale[idx]);
        }
        const float sc = scale_q * ks * (float)(2 * pop - head_dim);
        if (sc > st.m) {
            const float f = (st.m == -INFINITY) ? 0.0f : __expf(st.m - sc);
            st.z = st.z * f + 1.0f;
            st.w = st.w * f + sc;
            st.m = sc;
        } else {
            const float e = __expf(sc - st.m);
            st.z += e;
            st.w += e * sc;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        EntState o{__shfl_xor_sync(0xffffffffu, st.m, off), __shfl_xor_sync(0xffffffffu, st.z, off),
                   __shfl_xor_sync(0xffffffffu, st.w, off)};
        st = ent_merge(st, o);
    }
    if (lane == 0) s_part[warp] = st;
    __syncthreads();
    if (tid == 0) {
        EntState t = s_part[0];
        for (int w = 1; w < kEntThreads / 32; ++w) t = ent_merge(t, s_part[w]);
        const float log_z = logf(t.z) + t.m;
        out[h] = log_z - t.w / fmaxf(t.z, 1e-12f);
    }
}

__global__ void k_adaptive_select(const float* __restrict__ ent, uint8_t* __restrict__ modes, int n, float thr) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) modes[i] = (ent[i] >= thr) ? 0 : 1;
}

}  // namespace bc

using namespace bc;

#define BC_DISPATCH_NW_E(d, CALL)                            \
    switch ((d) / 32) {                                      \
        case 1: { constexpr int NW = 1; CALL; break; }      \
        case 2: { constexpr int NW = 2; CALL; break; }      \
        case 3: { constexpr int NW = 3; CALL; break; }      \
        case 4: { constexpr int NW = 4; CALL; break; }      \
        case 5: { constexpr int NW = 5; CALL; break; }      \
        case 6: { constexpr int NW = 6; CALL; break; }      \
        case 7: { constexpr int NW = 7; CALL; break; }      \
        case 8: { constexpr int NW = 8; CALL; break; }      \
        default: return BC_ERR_HEAD_DIM;                    \
    }

extern "C" {

size_t bc_entropy_workspace_bytes(int batch, int n_heads, int seq_len) {
    (void)batch;
    (void)n_heads;
    (void)seq_len;
    return 0;
}

int bc_compute_head_entropy(const void* q, const void* k_bin, float* entropy, int batch, int n_heads, int seq_len,
                            int head_dim, void* workspace, size_t workspace_bytes, void* stream) {
    (void)workspace;
    (void)workspace_bytes;
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (batch < 0 || n_heads < 0 || seq_len < 0) return BC_ERR_ARG;
    const int n = batch * n_heads;
    if (n == 0) return BC_OK;
    if (!q || !k_bin || !entropy) return BC_ERR_ARG;
    if (!bc_aligned(k_bin, 4)) return BC_ERR_ALIGN;
    BC_DISPATCH_NW_E(head_dim, (k_head_entropy<NW, true><<<n, kEntThreads, 0, (cudaStream_t)stream>>>(
                                    (const __half*)q, (const uint8_t*)k_bin, nullptr, entropy, seq_len,
                                    (int64_t)seq_len, head_dim)));
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_head_entropy_planes(const void* q, bc_kv_planes K, float* entropy, int n_heads, int seq_len,
                           int64_t kv_stride, int head_dim, void* stream) {
    if (!bc_valid_head_dim(head_dim)) return BC_ERR_HEAD_DIM;
    if (n_heads < 0 || seq_len < 0 || kv_stride < seq_len) return BC_ERR_ARG;
    if (n_heads == 0) return BC_OK;
    if (!q || !K.sign || !K.bscale || !entropy) return BC_ERR_ARG;
    BC_DISPATCH_NW_E(head_dim, (k_head_entropy<NW, false><<<n_heads, kEntThreads, 0, (cudaStream_t)stream>>>(
                                    (const __half*)q, (const uint8_t*)K.sign, (const __half*)K.bscale, entropy,
                                    seq_len, kv_stride, head_dim)));
    BC_LAUNCH_CHECK();
    return BC_OK;
}

int bc_adaptive_select(const float* entropy, uint8_t* modes, int batch, int n_heads, float threshold,
                       void* stream) {
    if (batch < 0 || n_heads < 0) return BC_ERR_ARG;
    const int n = batch * n_heads;
    if (n == 0) return BC_OK;
    if (!entropy || !modes) return BC_ERR_ARG;
    k_adaptive_select<<<(n + 127) / 128, 128, 0, (cudaStream_t)stream>>>(entropy, modes, n, threshold);
    BC_LAUNCH_CHECK();
    return BC_OK;
}

}  // extern "C"
