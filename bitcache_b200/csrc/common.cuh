// Shared device/host definitions for the bitcache B200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "bitcache_b200.h"

namespace bc {

// ---------------------------------------------------------------------------
// Reference record formats (byte-compatible with the reference structs).
//   BinaryVec   : uint32 words[8]; __half scale;          sizeof 36, align 4
//   ResidualVec : uint8 nibbles[128]; __half scale;        sizeof 130, align 2
// (binary_encode.cuh:13-18, residual.cuh:11-16 of the reference.)
// ---------------------------------------------------------------------------
constexpr int kMaxHeadDim = 256;
constexpr int kBinRecBytes = 36;
constexpr int kBinScaleOff = 32;
constexpr int kResRecBytes = 130;
constexpr int kResScaleOff = 128;

// Nibble plane layout: offset-binary codes (each nibble holds code + 8, so
// the reference's two's-complement byte XOR 0x88), interleaved in blocks of 8
// positions.  Chunk c (16 bytes = 32 dims, element 2i in the low nibble of
// byte i) of plane row p
// lives at byte (p/8)*(8*d/2) + c*128 + (p%8)*16, so one block of 8 rows is
// d/32 runs of 8 consecutive 16-byte chunks.  Tiles that start at a multiple
// of 8 rows are still contiguous byte ranges, and both the key-per-lane and
// the chunk-per-lane readers of the decode kernel hit distinct shared-memory
// banks.
__host__ __device__ __forceinline__ int64_t nib_chunk_offset(int64_t row, int c, int d) {
    return (row >> 3) * (int64_t)(4 * d) + (int64_t)c * 128 + (row & 7) * 16;
}

// Which dims a chunk holds.  At head dims 64, 128 and 256 the order is "by
// bit": every nibble byte holds bits t and t + 4 (t < 4) of one sign byte b,
// i.e. dims 8b + t (low nibble) and 8b + t + 4 (high nibble), placed so that
// the bytes of one 16-byte chunk line up with one 16-byte window of the sign
// row (the decode kernel's tensor-core value phase then gives a dim's sign
// bit and its code the same accumulator row):
//   d = 128: byte j of chunk c is (b = j, t = c);
//   d = 256: byte j of chunk c is (b = 16 (c / 4) + j, t = c % 4);
//   d = 64:  byte j of chunk c is (b = j % 8, t = 2c + j / 8) (the sign row is
//            8 bytes, so one 16-byte chunk holds two bits of each sign byte).
// Other head dims keep the reference's element order: byte j of chunk c holds
// dims 32c + 2j (low) and 32c + 2j + 1 (high).  The values are the
// reference's; only their places differ (the record converters permute).
__host__ __device__ constexpr bool nib_by_bit(int d) { return d == 64 || d == 128 || d == 256; }
__host__ __device__ constexpr int nib_dim(int d, int c, int j, int hi) {
    return d == 128   ? 8 * j + c + 4 * hi
           : d == 256 ? 128 * (c / 4) + 8 * j + (c % 4) + 4 * hi
           : d == 64  ? 8 * (j % 8) + 2 * c + j / 8 + 4 * hi
                      : 32 * c + 2 * j + hi;
}
// Inverse of the by-bit order: the chunk and the byte within it that hold
// bits t and t + 4 of sign byte b (t < 4).
__host__ __device__ constexpr int nib_byte_chunk(int d, int b, int t) {
    return d == 128 ? t : d == 256 ? 4 * (b / 16) + t : t / 2;
}
__host__ __device__ constexpr int nib_byte_index(int d, int b, int t) {
    return d == 128 ? b : d == 256 ? b % 16 : 8 * (t % 2) + b;
}

// ---------------------------------------------------------------------------
// Device-side error word.  Kernels never trap: a bounded wait that gives up
// ORs a code into the error word (defined once, in decode.cu, whose kernels
// own every bounded wait) and the kernel returns; bc_get_device_error() reads
// and clears it from the host.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void raise_device_error(unsigned int* word, unsigned int code) { atomicOr(word, code); }

// Iteration cap for every spin on an mbarrier or a flag.  try_wait already
// suspends for a hardware-defined interval per attempt, so this bounds a wait
// to well under a minute while never triggering on a healthy GPU.
constexpr uint32_t kSpinLimit = 1u << 24;

// ---------------------------------------------------------------------------
// mbarrier + 1-D bulk copy (TMA) helpers.  No multicast anywhere.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: true when the phase completed, false after kSpinLimit tries.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < kSpinLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// 1-D bulk global->shared copy completing on an mbarrier.  dst, src and bytes
// must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of a global range into L2 (no shared memory involved).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100).  Written without .ftz so that denormal
// operands are honoured: the V accumulation feeds sign bits and INT4 codes in
// as denormal bit patterns (value = pattern * 2^-149) and rescales them with
// power-of-two coefficients, which is exact.
// ---------------------------------------------------------------------------
struct f2 {
    float x, y;
};

__device__ __forceinline__ void ffma2(f2& acc, f2 a, f2 b) {
    unsigned long long r, ua, ub, uc;
    ua = *reinterpret_cast<unsigned long long*>(&a);
    ub = *reinterpret_cast<unsigned long long*>(&b);
    uc = *reinterpret_cast<unsigned long long*>(&acc);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(ua), "l"(ub), "l"(uc));
    acc = *reinterpret_cast<f2*>(&r);
}

__device__ __forceinline__ void fmul2(f2& acc, f2 a) {
    unsigned long long r, ua, uc;
    ua = *reinterpret_cast<unsigned long long*>(&a);
    uc = *reinterpret_cast<unsigned long long*>(&acc);
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(uc), "l"(ua));
    acc = *reinterpret_cast<f2*>(&r);
}

__device__ __forceinline__ float bits_f(uint32_t u) { return __uint_as_float(u); }

// Exact power of two 2^e for e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

__device__ __forceinline__ int dp4a_us(uint32_t a_u8, uint32_t b_s8, int c) {
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a_u8), "r"(b_s8), "r"(c));
    return r;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a_u8, uint32_t b_u8, int c) {
    int r;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a_u8), "r"(b_u8), "r"(c));
    return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Streaming 16-byte read-only global load.
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

}  // namespace bc

// Device address of the library's error word on the current device (defined
// in decode.cu), for kernels of other translation units.
unsigned int* bc_device_error_ptr();

// Record-layout attention for the C++ launchers (decode.cu): split-K scratch
// in a fixed 4 MiB array of the library instead of a caller workspace, with
// fewer splits when the partials would not fit.  Calls that overlap on the GPU
// share that array and race.  Allocates nothing.
int bc_record_attention_fixed_scratch(const void* q, const void* k_bin, const void* k_res, const void* v_bin,
                                      const void* v_res, void* out, int batch, int n_heads, int seq_len, int head_dim,
                                      bool compensated, void* stream);

// ---------------------------------------------------------------------------
// Host-side helpers shared by the entry points.
// ---------------------------------------------------------------------------
#define BC_LAUNCH_CHECK()                                  \
    do {                                                   \
        cudaError_t _e = cudaGetLastError();               \
        if (_e != cudaSuccess) return BC_ERR_CUDA_BASE + (int)_e; \
    } while (0)

static inline bool bc_valid_head_dim(int d) { return d > 0 && d % 32 == 0 && d <= bc::kMaxHeadDim; }
static inline bool bc_aligned(const void* p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }
