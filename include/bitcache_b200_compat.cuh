// bitcache_b200 -- C++ host API with the reference's launcher signatures.
//
// Drop-in replacement for the launch_* functions and record structs declared
// in the reference's src/*.cuh (anishesg/bitcache).  The record structs are
// byte-identical to the reference's, so buffers can be shared with code built
// against the reference headers.  Implemented in libbitcache_b200.so on top of
// the C ABI in bitcache_b200.h.
//
// Differences from the reference, all on invalid input or error paths:
//  - head_dim is checked at run time (the reference asserts); a bad head_dim or
//    a failed launch is reported through bc_last_status() instead of aborting.
//  - The attention launchers guard batch*n_heads (the reference kernels need
//    every buffer padded to a multiple of 32 rows).
//  - Like the reference's, no launcher allocates.  The attention launchers keep
//    their split-K partials in a fixed 4 MiB array inside the library (held by
//    every GPU that loads it until exit) and plan fewer splits for shapes whose
//    partials would not fit.  Attention launches that overlap on the GPU
//    (concurrent streams) share that array and race: serialise them, or use
//    the C ABI variants, which take a caller workspace.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "bitcache_b200.h"

#define WORDS_PER_VEC(head_dim) (((head_dim) + 31) / 32)
#define MAX_HEAD_DIM 256

// reference binary_encode.cuh:13-18
struct BinaryVec {
    uint32_t words[MAX_HEAD_DIM / 32];
    __half scale;
};

// reference residual.cuh:11-16
struct ResidualVec {
    uint8_t nibbles[MAX_HEAD_DIM / 2];
    __half scale;
};

// reference adaptive_precision.cuh:28-31
enum class PrecisionMode : uint8_t {
    BINARY = 0,
    COMPENSATED = 1,
};

static_assert(sizeof(BinaryVec) == 36, "BinaryVec layout");
static_assert(sizeof(ResidualVec) == 130, "ResidualVec layout");

// Status of the most recent launch_* call on this host thread (BC_OK on success).
int bc_last_status();

// reference binary_encode.cuh:26-32
void launch_binary_encode(const __half* src, BinaryVec* out, int n_vecs, int head_dim, cudaStream_t stream = 0);
// reference residual.cuh:26-33
void launch_residual_encode(const __half* src, const BinaryVec* binary, ResidualVec* out, int n_vecs, int head_dim,
                            cudaStream_t stream = 0);
// reference binary_attention.cuh:15-25
void launch_binary_attention(const __half* Q, const BinaryVec* K_bin, const BinaryVec* V_bin, __half* out, int batch,
                             int n_heads, int seq_len, int head_dim, cudaStream_t stream = 0);
// reference compensated_attention.cuh:16-28
void launch_compensated_attention(const __half* Q, const BinaryVec* K_bin, const ResidualVec* K_res,
                                  const BinaryVec* V_bin, const ResidualVec* V_res, __half* out, int batch,
                                  int n_heads, int seq_len, int head_dim, cudaStream_t stream = 0);
// reference online_encode.cuh:15-25
void launch_online_encode_token(const __half* kv, BinaryVec* binary_cache, ResidualVec* residual_cache, int batch,
                                int n_heads, int head_dim, int current_len, int max_seq, cudaStream_t stream = 0);
// reference adaptive_precision.cuh:14-23
void launch_compute_head_entropy(const __half* Q, const BinaryVec* K_bin, float* entropy_out, int batch, int n_heads,
                                 int seq_len, int head_dim, cudaStream_t stream = 0);
// reference adaptive_precision.cuh:42-49
void launch_adaptive_select(const float* entropy, PrecisionMode* modes_out, int batch, int n_heads,
                            float entropy_threshold, cudaStream_t stream = 0);
