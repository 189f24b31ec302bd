// C++ launchers with the reference signatures (include/bitcache_b200_compat.cuh),
// implemented on the C ABI.
#include "bitcache_b200_compat.cuh"

namespace {
thread_local int t_last_status = BC_OK;

// Split-K scratch from the stream-ordered pool: zero-filled, used, released on
// the same stream, so concurrent streams never share it.
template <typename F>
int with_workspace(size_t bytes, cudaStream_t stream, F&& fn) {
    if (bytes == 0) return fn(nullptr, 0);
    void* ws = nullptr;
    cudaError_t e = cudaMallocAsync(&ws, bytes, stream);
    if (e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)e;
    e = cudaMemsetAsync(ws, 0, bytes, stream);
    int rc = (e == cudaSuccess) ? fn(ws, bytes) : BC_ERR_CUDA_BASE + (int)e;
    cudaFreeAsync(ws, stream);
    return rc;
}
}  // namespace

int bc_last_status() { return t_last_status; }

void launch_binary_encode(const __half* src, BinaryVec* out, int n_vecs, int head_dim, cudaStream_t stream) {
    t_last_status = bc_binary_encode(src, out, n_vecs, head_dim, stream);
}

void launch_residual_encode(const __half* src, const BinaryVec* binary, ResidualVec* out, int n_vecs, int head_dim,
                            cudaStream_t stream) {
    t_last_status = bc_residual_encode(src, binary, out, n_vecs, head_dim, stream);
}

void launch_binary_attention(const __half* Q, const BinaryVec* K_bin, const BinaryVec* V_bin, __half* out, int batch,
                             int n_heads, int seq_len, int head_dim, cudaStream_t stream) {
    const size_t need = bc_attention_workspace_bytes(batch, n_heads, seq_len, head_dim);
    t_last_status = with_workspace(need, stream, [&](void* ws, size_t n) {
        return bc_binary_attention(Q, K_bin, V_bin, out, batch, n_heads, seq_len, head_dim, ws, n, stream);
    });
}

void launch_compensated_attention(const __half* Q, const BinaryVec* K_bin, const ResidualVec* K_res,
                                  const BinaryVec* V_bin, const ResidualVec* V_res, __half* out, int batch,
                                  int n_heads, int seq_len, int head_dim, cudaStream_t stream) {
    const size_t need = bc_attention_workspace_bytes(batch, n_heads, seq_len, head_dim);
    t_last_status = with_workspace(need, stream, [&](void* ws, size_t n) {
        return bc_compensated_attention(Q, K_bin, K_res, V_bin, V_res, out, batch, n_heads, seq_len, head_dim, ws, n,
                                        stream);
    });
}

void launch_online_encode_token(const __half* kv, BinaryVec* binary_cache, ResidualVec* residual_cache, int batch,
                                int n_heads, int head_dim, int current_len, int max_seq, cudaStream_t stream) {
    t_last_status = bc_online_encode_token(kv, binary_cache, residual_cache, batch, n_heads, head_dim, current_len,
                                           max_seq, stream);
}

void launch_compute_head_entropy(const __half* Q, const BinaryVec* K_bin, float* entropy_out, int batch, int n_heads,
                                 int seq_len, int head_dim, cudaStream_t stream) {
    const size_t need = bc_entropy_workspace_bytes(batch, n_heads, seq_len);
    t_last_status = with_workspace(need, stream, [&](void* ws, size_t n) {
        return bc_compute_head_entropy(Q, K_bin, entropy_out, batch, n_heads, seq_len, head_dim, ws, n, stream);
    });
}

void launch_adaptive_select(const float* entropy, PrecisionMode* modes_out, int batch, int n_heads,
                            float entropy_threshold, cudaStream_t stream) {
    t_last_status = bc_adaptive_select(entropy, reinterpret_cast<uint8_t*>(modes_out), batch, n_heads,
                                       entropy_threshold, stream);
}
