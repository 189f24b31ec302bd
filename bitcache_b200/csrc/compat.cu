// C++ launchers with the reference signatures (include/bitcache_b200_compat.cuh),
// implemented on the C ABI.  Like the reference's launchers they allocate
// nothing: the attention launchers keep their split-K partials in a fixed
// array of the library (bc_record_attention_fixed_scratch).
#include "bitcache_b200_compat.cuh"
#include "common.cuh"

namespace {
thread_local int t_last_status = BC_OK;
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
    t_last_status = bc_record_attention_fixed_scratch(Q, K_bin, nullptr, V_bin, nullptr, out, batch, n_heads, seq_len,
                                                      head_dim, false, stream);
}

void launch_compensated_attention(const __half* Q, const BinaryVec* K_bin, const ResidualVec* K_res,
                                  const BinaryVec* V_bin, const ResidualVec* V_res, __half* out, int batch,
                                  int n_heads, int seq_len, int head_dim, cudaStream_t stream) {
    t_last_status = bc_record_attention_fixed_scratch(Q, K_bin, K_res, V_bin, V_res, out, batch, n_heads, seq_len,
                                                      head_dim, true, stream);
}

void launch_online_encode_token(const __half* kv, BinaryVec* binary_cache, ResidualVec* residual_cache, int batch,
                                int n_heads, int head_dim, int current_len, int max_seq, cudaStream_t stream) {
    t_last_status = bc_online_encode_token(kv, binary_cache, residual_cache, batch, n_heads, head_dim, current_len,
                                           max_seq, stream);
}

void launch_compute_head_entropy(const __half* Q, const BinaryVec* K_bin, float* entropy_out, int batch, int n_heads,
                                 int seq_len, int head_dim, cudaStream_t stream) {
    // the entropy kernel needs no scratch (bc_entropy_workspace_bytes is 0)
    t_last_status =
        bc_compute_head_entropy(Q, K_bin, entropy_out, batch, n_heads, seq_len, head_dim, nullptr, 0, stream);
}

void launch_adaptive_select(const float* entropy, PrecisionMode* modes_out, int batch, int n_heads,
                            float entropy_threshold, cudaStream_t stream) {
    t_last_status = bc_adaptive_select(entropy, reinterpret_cast<uint8_t*>(modes_out), batch, n_heads,
                                       entropy_threshold, stream);
}
