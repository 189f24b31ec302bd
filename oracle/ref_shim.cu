// C-ABI shim over the reference bitcache launchers -- TEST INFRASTRUCTURE ONLY.
//
// Compiled together with the reference's own kernel sources (src/*.cu of
// anishesg/bitcache, taken from where they lie, never copied) into
// oracle/_ref/libbitcache_ref.so by oracle/build.py.  Tests load it through
// ctypes to run the reference kernels on the same inputs as the B200 kernels.
//
// The reference attention kernels have no `bh < batch*n_heads` guard
// (compensated_attention.cu:52, binary_attention.cu:17): callers must pad every
// per-(batch, head) buffer to a multiple of 32 rows.  The wrappers below only
// forward; the Python side (oracle/refgpu.py) does the padding.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include "binary_encode.cuh"
#include "residual.cuh"
#include "binary_attention.cuh"
#include "compensated_attention.cuh"
#include "online_encode.cuh"
#include "adaptive_precision.cuh"
#include "reference_attention.cuh"

extern "C" {

int ref_sizeof_binary_vec(void) { return (int)sizeof(BinaryVec); }
int ref_sizeof_residual_vec(void) { return (int)sizeof(ResidualVec); }

int ref_binary_encode(const void* src, void* out, int n_vecs, int head_dim, void* stream) {
    launch_binary_encode((const __half*)src, (BinaryVec*)out, n_vecs, head_dim, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_residual_encode(const void* src, const void* bin, void* out, int n_vecs, int head_dim, void* stream) {
    launch_residual_encode((const __half*)src, (const BinaryVec*)bin, (ResidualVec*)out, n_vecs, head_dim,
                           (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_binary_attention(const void* q, const void* kb, const void* vb, void* out, int batch, int n_heads,
                         int seq_len, int head_dim, void* stream) {
    launch_binary_attention((const __half*)q, (const BinaryVec*)kb, (const BinaryVec*)vb, (__half*)out, batch,
                            n_heads, seq_len, head_dim, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_compensated_attention(const void* q, const void* kb, const void* kr, const void* vb, const void* vr,
                              void* out, int batch, int n_heads, int seq_len, int head_dim, void* stream) {
    launch_compensated_attention((const __half*)q, (const BinaryVec*)kb, (const ResidualVec*)kr,
                                 (const BinaryVec*)vb, (const ResidualVec*)vr, (__half*)out, batch, n_heads,
                                 seq_len, head_dim, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_online_encode_token(const void* kv, void* bin, void* res, int batch, int n_heads, int head_dim,
                            int current_len, int max_seq, void* stream) {
    launch_online_encode_token((const __half*)kv, (BinaryVec*)bin, (ResidualVec*)res, batch, n_heads, head_dim,
                               current_len, max_seq, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_compute_head_entropy(const void* q, const void* kb, float* ent, int batch, int n_heads, int seq_len,
                             int head_dim, void* stream) {
    launch_compute_head_entropy((const __half*)q, (const BinaryVec*)kb, ent, batch, n_heads, seq_len, head_dim,
                                (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_adaptive_select(const float* ent, void* modes, int batch, int n_heads, float thr, void* stream) {
    launch_adaptive_select(ent, (PrecisionMode*)modes, batch, n_heads, thr, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_reference_attention(const void* q, const void* k, const void* v, void* out, int batch, int n_heads,
                            int seq_len, int head_dim, void* stream) {
    launch_reference_attention((const __half*)q, (const __half*)k, (const __half*)v, (__half*)out, batch, n_heads,
                               seq_len, head_dim, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

}  // extern "C"
