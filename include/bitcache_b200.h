/*
 * bitcache_b200 -- C ABI of the B200 (sm_100a) implementation of bitcache's
 * quantized decode-attention path.
 *
 * Plain C: raw device pointers, sizes and a CUDA stream passed as void*
 * (cudaStream_t; NULL = legacy default stream).  Every entry point returns an
 * int status (BC_OK = 0).  Launches are asynchronous; none synchronises the
 * host.  No entry point allocates memory unless its comment says so; ops that
 * need scratch take a caller-provided workspace whose size is given by the
 * matching *_workspace_bytes() query.  A workspace holds one ticket counter
 * per (slot, head group) followed by split partials; every completed call
 * returns its counters to zero.  Zero-fill a workspace before its first use
 * and again before using it with a different (n_slots, group) -- another
 * shape's partials may overlap this shape's counters -- or after a
 * BC_DEVERR_TIMEOUT.  Calls that overlap on the GPU must not share one.
 *
 * Two storage formats:
 *  - reference records: arrays of the reference's BinaryVec (36 B) and
 *    ResidualVec (130 B) structs, byte-compatible with anishesg/bitcache
 *    (src/binary_encode.cuh:13-18, src/residual.cuh:11-16).  The bc_* ops
 *    below that take "record" pointers are drop-ins for the reference
 *    launchers named beside them.
 *  - planes (native): per K or V cache, four 16-byte-aligned arrays indexed
 *    [slot][position] with a row stride kv_stride (positions per slot):
 *        sign   uint32 [slots][kv_stride][head_dim/32]   bit i%32 of word i/32 = (x_i >= 0)
 *        nib    uint8  [slots][kv_stride][head_dim/2]    INT4 residual codes stored offset-binary
 *               (each nibble holds code + 8), interleaved in blocks of 8 positions: the
 *               16-byte chunk c of plane row r = slot*kv_stride + pos starts at byte
 *               (r/8)*(4*head_dim) + c*128 + (r%8)*16.  At head dims 64, 128 and 256
 *               every byte holds the dims of bits t and t+4 (t < 4) of one sign byte b,
 *               8b + t (low nibble) and 8b + t + 4 (high nibble); byte j of chunk c is
 *                 head_dim 128:   b = j,               t = c
 *                 head_dim 256:   b = 16*(c/4) + j,    t = c % 4
 *                 head_dim 64:    b = j % 8,           t = 2c + j/8
 *               (one chunk lines up with one 16-byte window of the sign row).  Other
 *               head dims keep the reference's element order: byte j of chunk c holds
 *               dims 32c + 2j (low) and 32c + 2j + 1 (high) (the reference's byte XOR 0x88).
 *        bscale fp16   [slots][kv_stride]                mean |x| (binary scale)
 *        rscale fp16   [slots][kv_stride]                residual absmax
 *    5*head_dim/8 + 4 bytes per vector (84 B at head_dim 128).  The field
 *    values are bit-identical to the reference records; only the layout differs.
 */
#ifndef BITCACHE_B200_H
#define BITCACHE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define BC_OK 0
#define BC_ERR_HEAD_DIM 1    /* head_dim not a multiple of 32 in [32, 256] */
#define BC_ERR_ARG 2         /* negative/zero size, null pointer, bad mode */
#define BC_ERR_ALIGN 3       /* pointer not 16-byte aligned, or kv_stride % 8 != 0 */
#define BC_ERR_WORKSPACE 4   /* workspace smaller than the *_workspace_bytes() query */
#define BC_ERR_UNSUPPORTED 5 /* shape outside the compiled kernel set (e.g. GQA group) */
#define BC_ERR_TOO_LARGE 6   /* size exceeds a documented fixed maximum */
#define BC_ERR_CUDA_BASE 1000 /* BC_ERR_CUDA_BASE + cudaError_t of a failed launch/call */

/* device-side error bits, read with bc_get_device_error() */
#define BC_DEVERR_TIMEOUT 1u /* a bounded wait in a kernel gave up; outputs are invalid */
#define BC_DEVERR_PAGE 2u    /* a block-table entry named a page outside the pool; that tile
                                was not read or written and the outputs are invalid */

/* residual modes for the encoders */
#define BC_RES_NONE 0       /* binary only: sign + bscale */
#define BC_RES_FP16_SCALE 1 /* residual against the fp16-rounded scale (reference residual.cu:28) */
#define BC_RES_FP32_SCALE 2 /* residual against the fp32 scale (reference online_encode.cu:74) */

/* attention modes */
#define BC_MODE_BINARY 0      /* xnor-popcount scores, sign*scale values (binary_attention.cu) */
#define BC_MODE_COMPENSATED 1 /* + INT4 residual in scores and values (compensated_attention.cu) */

const char* bc_status_string(int status);
/* Reads (and when clear != 0 resets) the device error word of the current device.
 * Synchronises the current device. */
unsigned int bc_get_device_error(int clear);

/* ====================================================================== */
/* Reference-record operations (drop-ins for the reference launchers)     */
/* ====================================================================== */

/* sizeof(BinaryVec) = 36 and sizeof(ResidualVec) = 130, as
 * sizeof_binary_vec / sizeof_residual_vec, reference torch_binding.cpp:165-166. */
int64_t bc_sizeof_binary_vec(void);
int64_t bc_sizeof_residual_vec(void);

/* launch_binary_encode, reference binary_encode.cuh:26-32 / binary_encode.cu:62-80.
 * src fp16 [n_vecs][head_dim] -> BinaryVec[n_vecs].  Unused words and padding are zeroed. */
int bc_binary_encode(const void* src, void* out_binvec, int64_t n_vecs, int head_dim, void* stream);

/* launch_residual_encode, reference residual.cuh:26-33 / residual.cu:80-98.
 * The residual is taken against the binary record's stored (fp16) scale and sign bits. */
int bc_residual_encode(const void* src, const void* binvec, void* out_resvec, int64_t n_vecs, int head_dim,
                       void* stream);

/* launch_online_encode_token, reference online_encode.cuh:15-25 / online_encode.cu:122-149.
 * kv fp16 [batch*n_heads][head_dim] written at record slot*max_seq + current_len % max_seq.
 * res_cache may be NULL (binary-only cache). */
int bc_online_encode_token(const void* kv, void* bin_cache, void* res_cache, int batch, int n_heads,
                           int head_dim, int current_len, int max_seq, void* stream);

/* launch_binary_attention, reference binary_attention.cuh:15-25, and
 * launch_compensated_attention, reference compensated_attention.cuh:16-28.
 * q/out fp16 [batch*n_heads][head_dim]; records [batch*n_heads][seq_len].
 * Unlike the reference kernels these guard batch*n_heads (no 32-row padding needed). */
size_t bc_attention_workspace_bytes(int batch, int n_heads, int seq_len, int head_dim);
int bc_binary_attention(const void* q, const void* k_bin, const void* v_bin, void* out, int batch, int n_heads,
                        int seq_len, int head_dim, void* workspace, size_t workspace_bytes, void* stream);
int bc_compensated_attention(const void* q, const void* k_bin, const void* k_res, const void* v_bin,
                             const void* v_res, void* out, int batch, int n_heads, int seq_len, int head_dim,
                             void* workspace, size_t workspace_bytes, void* stream);

/* launch_compute_head_entropy, reference adaptive_precision.cuh:14-23:
 * entropy of the softmax over binary scores (no 1/sqrt(d)) per (batch, head). */
size_t bc_entropy_workspace_bytes(int batch, int n_heads, int seq_len);
int bc_compute_head_entropy(const void* q, const void* k_bin, float* entropy, int batch, int n_heads,
                            int seq_len, int head_dim, void* workspace, size_t workspace_bytes, void* stream);

/* launch_adaptive_select, reference adaptive_precision.cuh:42-49:
 * modes[i] = entropy[i] >= threshold ? 0 (BINARY) : 1 (COMPENSATED). */
int bc_adaptive_select(const float* entropy, uint8_t* modes, int batch, int n_heads, float threshold,
                       void* stream);

/* ====================================================================== */
/* Native plane layout                                                    */
/* ====================================================================== */

typedef struct bc_kv_planes {
    void* sign;   /* uint32 [slots][kv_stride][head_dim/32] */
    void* nib;    /* uint8, interleaved as above             (NULL for binary-only caches) */
    void* bscale; /* fp16   [slots][kv_stride] */
    void* rscale; /* fp16   [slots][kv_stride]              (NULL for binary-only caches) */
} bc_kv_planes;

/* Prefill encode (binary_encode.cu + residual.cu, or online_encode.cu arithmetic with
 * BC_RES_FP32_SCALE) of src fp16 [n_slots][seq_len][head_dim] into plane rows
 * slot*kv_stride + s.  Nothing in the reference fuses these two passes. */
int bc_encode_planes(const void* src, bc_kv_planes out, int n_slots, int seq_len, int64_t kv_stride,
                     int head_dim, int residual_mode, void* stream);

/* Decode-step append: online_encode.cu arithmetic (BC_RES_FP32_SCALE) or binary only, for
 * one K and one V token per slot (k, v fp16 [n_slots][head_dim]) at plane position pos, in one
 * launch.  The reference needs two launches (one per tensor, bitcache/__init__.py:104-111). */
int bc_append_kv(const void* k, const void* v, bc_kv_planes K, bc_kv_planes V, int n_slots, int head_dim,
                 int64_t kv_stride, int64_t pos, int residual_mode, void* stream);

/* Fused split-K decode attention over plane caches (compensated_attention.cu:42-109 or
 * binary_attention.cu:8-82 arithmetic) with grouped-query heads: query head
 * slot*group + g reads KV slot `slot`, keys [0, seq_len).  q fp16 [n_slots*group][head_dim].
 * Output: out fp16 [n_slots*group][head_dim] when out != NULL, and/or the per-head
 * log-sum-exp partial triples when partial != NULL: partial[h*(head_dim+2) + {0: m, 1: l,
 * 2..: o}] with m = max score (natural log units), l = sum exp(score - m),
 * o = sum exp(score - m) * v (unnormalised); merge with bc_lse_merge.
 * Requirements: kv_stride % 8 == 0, seq_len <= kv_stride, plane pointers 16-byte aligned,
 * group in {1, 2, 4, 8}. */
size_t bc_decode_workspace_bytes(int n_slots, int group, int seq_len, int head_dim);
int bc_decode_attention(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial, int n_slots,
                        int group, int seq_len, int64_t kv_stride, int head_dim, int mode, void* workspace,
                        size_t workspace_bytes, void* stream);

/* bc_decode_attention plus, in the same pass over the cache, the reference's
 * compute_head_entropy (adaptive_precision.cu:13-130; launch_compute_head_entropy,
 * adaptive_precision.cuh:14-23) for every query head: entropy[h] = H of the
 * softmax over the binary scores scale_q*scale_k*(2*matches - d) without
 * 1/sqrt(d), scale_q the query's mean |q| in the reference's tree order.
 * The reference needs a separate pass over K for it. fp32 [n_slots*group].
 * Workspace as bc_decode_workspace_bytes. */
int bc_decode_attention_entropy(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial,
                                float* entropy, int n_slots, int group, int seq_len, int64_t kv_stride, int head_dim,
                                int mode, void* workspace, size_t workspace_bytes, void* stream);

/* Fused decode step: bc_append_kv of new_k / new_v (fp16 [n_slots][head_dim]) at plane
 * position append_pos with append_res arithmetic, then bc_decode_attention over keys
 * [0, seq_len), in ONE launch.  Replaces the reference's BitCache.append followed by
 * BitCache.attend (bitcache/__init__.py:95-148: two online_encode_token launches and one
 * attention launch).  Results are identical to bc_append_kv + bc_decode_attention: the
 * planes receive the same bytes, and the appended row is attended from the encoder's
 * output, not re-read.  append_pos = -1 appends nothing (plain decode); otherwise
 * 0 <= append_pos < seq_len, and compensated attention needs append_res != BC_RES_NONE.
 * q, new_k, new_v and out may point to pinned (page-locked) host memory: with unified
 * addressing the kernel reads the step's inputs and writes its output over the host link
 * itself, so a host-driven decode loop needs no separate copies.  Host inputs are read
 * before the kernel waits for the previous one in the stream (programmatic dependent
 * launch), so they must not be written by work queued ahead of this call.  Pageable
 * host pointers are rejected with BC_ERR_ARG.
 * Workspace as bc_decode_workspace_bytes. */
int bc_decode_step(const void* q, const void* new_k, const void* new_v, bc_kv_planes K, bc_kv_planes V, void* out,
                   float* partial, int n_slots, int group, int seq_len, int64_t kv_stride, int head_dim, int mode,
                   int append_pos, int append_res, void* workspace, size_t workspace_bytes, void* stream);

/* ---- paged caches ----------------------------------------------------
 * A paged cache is a pool of pages, each page_size positions of one slot,
 * stored as planes with n_slots = n_pages and kv_stride = page_size (so page
 * p is plane rows [p*page_size, (p+1)*page_size)).  A block table maps the
 * logical page j of slot s to its physical page:
 *     pages[s*max_pages + j]   (int32, device memory)
 * Logical position pos of slot s lives in plane row
 *     pages[s*max_pages + pos/page_size]*page_size + pos%page_size.
 * page_size must be a multiple of 128 (the decode tile), so a tile never
 * straddles two pages.  Page ids are checked in the kernels: an id outside
 * [0, n_pages) is not dereferenced; the kernel raises BC_DEVERR_PAGE instead.
 * The reference's BitCache is a contiguous ring (bitcache/__init__.py:76-82);
 * the north star's "paged binary+residual cache" is this layout. */
typedef struct bc_page_table {
    const int32_t* pages; /* device, [n_slots][max_pages] */
    int32_t max_pages;    /* row stride of pages (logical pages per slot) */
    int32_t page_size;    /* positions per page, a multiple of 128 */
    int32_t n_pages;      /* pages in the pool: valid ids are 0..n_pages-1 */
} bc_page_table;

/* bc_decode_step over a paged cache: optional append of new_k/new_v at logical
 * position append_pos (-1: none), then attention over logical keys [0, seq_len).
 * K and V are the pools (kv_stride = pt.page_size).  Results are bit-identical
 * to bc_decode_step on a contiguous cache holding the same rows. */
int bc_decode_step_paged(const void* q, const void* new_k, const void* new_v, bc_kv_planes K, bc_kv_planes V,
                         void* out, float* partial, bc_page_table pt, int n_slots, int group, int seq_len,
                         int head_dim, int mode, int append_pos, int append_res, void* workspace,
                         size_t workspace_bytes, void* stream);

/* bc_append_kv into a paged cache at logical position pos of every slot. */
int bc_append_kv_paged(const void* k, const void* v, bc_kv_planes K, bc_kv_planes V, bc_page_table pt, int n_slots,
                       int head_dim, int64_t pos, int residual_mode, void* stream);

/* ---- compact adaptive caches (per-position adaptive precision) ----------
 * bc_select_positions_topk: like bc_select_residual_topk, but one choice per
 * position for K and V together, keyed by the fp32 sum of the K and V keys;
 * writes keep (uint8 [n_slots][kv_stride], 1 = keep the residuals).
 * bc_compact_adaptive: stable partition of each slot's positions by keep into
 * new planes Kc, Vc: kept positions in order at sign/scale rows [0, n_keep)
 * and residual rows [0, n_keep) (residual row stride r_stride >= round8(n_keep));
 * the rest, binary only, at sign/scale rows [b0, b0 + seq_len - n_keep),
 * b0 = n_keep rounded up to 8 (sign/scale row stride c_stride).  Residuals of
 * the unkept positions are neither stored nor read: at head_dim 128 a decode
 * step then reads 0.25*84 + 0.75*18 = 34.5 B per vector at a 25% keep rate.
 * bc_decode_attention_adaptive: compensated attention over the kept keys and
 * binary attention over the rest, in one launch (their splits merge in the
 * kernel).  Equal, within the attention tolerance, to bc_decode_attention
 * with the unkept residuals zeroed (scale 0, codes 0).  Attention is
 * invariant to the key order, so the permutation needs no record.
 * No counterpart in the reference (its adaptive precision is per head). */
int bc_select_positions_topk(bc_kv_planes K, bc_kv_planes V, int n_slots, int seq_len, int64_t kv_stride,
                             int head_dim, int n_keep, uint8_t* keep, void* workspace, size_t workspace_bytes,
                             void* stream);
int bc_compact_adaptive(bc_kv_planes K, bc_kv_planes V, const uint8_t* keep, int n_slots, int seq_len,
                        int64_t kv_stride, int head_dim, int n_keep, bc_kv_planes Kc, bc_kv_planes Vc,
                        int64_t c_stride, int64_t r_stride, void* stream);
size_t bc_decode_adaptive_workspace_bytes(int n_slots, int group, int seq_len, int n_keep, int head_dim);
int bc_decode_attention_adaptive(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial,
                                 int n_slots, int group, int seq_len, int n_keep, int64_t kv_stride,
                                 int64_t res_stride, int head_dim, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* ---- sequence split over peer memory (one process per GPU) ------------
 * Each rank holds a contiguous slice of every slot's positions.  Instead of
 * an NCCL all-gather of the (m, l, o) triples followed by bc_lse_merge, the
 * last CTA of every (slot, head group) stores its triple directly into every
 * rank's exchange buffer over NVLink (plain peer stores of 64-bit words that
 * carry the value and the call's epoch, so no fence or flag is needed), waits
 * until every word it needs in its own buffer carries the epoch (a bounded
 * spin of spin_limit polls per word: BC_DEVERR_TIMEOUT after about a second
 * by default) and merges the world triples itself, so one launch per rank
 * yields the full output on every rank.  Setup (allocates, outside the decode
 * loop): bc_xchg_alloc on every rank, share the 64-byte bc_ipc_handle of each
 * buffer, bc_ipc_open the peers' handles.  Every rank calls
 * bc_decode_attention_xchg with the same n_slots, group, head_dim and epoch
 * (1, 2, 3, ...: one per call); ranks run on different GPUs.  A call whose
 * n_slots*group heads of head_dim do not fit buf_bytes returns BC_ERR_ARG.
 * Recovery after BC_DEVERR_TIMEOUT (a rank that never published): the output
 * of that call is invalid; clear the error (bc_get_device_error(1)), zero the
 * workspace, and continue with the next epoch once every rank is back.
 * No counterpart in the reference. */
typedef struct bc_xchg {
    void* bufs[8];       /* rank j's exchange buffer as mapped in this process (bufs[rank] = own) */
    int32_t world;       /* 1..8 */
    int32_t rank;
    uint32_t epoch;      /* call number, from 1, equal on every rank */
    uint32_t spin_limit; /* polls of one word before the wait gives up; 0 = default (about a second) */
    uint64_t buf_bytes;  /* bytes of each rank's buffer (all equal; bc_xchg_bytes at allocation) */
} bc_xchg;
size_t bc_xchg_bytes(int n_heads, int head_dim, int world);
int bc_xchg_alloc(size_t bytes, void** buf);          /* cudaMalloc + zero fill */
int bc_xchg_free(void* buf);
int bc_ipc_handle(const void* buf, void* handle_64_bytes);
int bc_ipc_open(const void* handle_64_bytes, void** buf);
int bc_ipc_close(void* buf);
int bc_decode_attention_xchg(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, int n_slots, int group,
                             int seq_len, int64_t kv_stride, int head_dim, int mode, bc_xchg x, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Allocation-free bc_decode_attention, for callers that cannot allocate
 * device memory where they run attention (an engine that reserves all of its
 * GPU memory at start-up and forbids allocation in the decode loop, or a
 * plugin whose host framework owns every device buffer).  No counterpart in
 * the reference (its launchers need no scratch).  Same arguments and results
 * as bc_decode_attention without the workspace: the split-K scratch is a
 * fixed array of bc_decode_noalloc_max_scratch_bytes() (4 MiB) inside the
 * library, held by every GPU that loads it until the process exits.  Shapes
 * whose bc_decode_workspace_bytes() exceeds that return BC_ERR_TOO_LARGE.
 * The first call on a device looks up the array's device address (with that
 * device current), so make it before any stream capture; the lookup is made
 * again when the device has a new context (after cudaDeviceReset).  All calls on a
 * device share the array: calls that overlap on the GPU (concurrent streams)
 * race and must be serialised by the caller.  Calls nothing that allocates. */
size_t bc_decode_noalloc_max_scratch_bytes(void);
int bc_decode_attention_noalloc(const void* q, bc_kv_planes K, bc_kv_planes V, void* out, float* partial,
                                int n_slots, int group, int seq_len, int64_t kv_stride, int head_dim, int mode,
                                void* stream);

/* Per-vector adaptive precision (no reference kernel; the reference adapts per head):
 * within each slot keep the INT4 residual of the n_keep vectors (of positions
 * [0, seq_len)) with the largest key fp32(rs*rs) * (float)sum_i code_i^2, ties
 * to the lower position.  keep (uint8 [slots][kv_stride], may be NULL when
 * apply != 0) receives 1 for kept vectors.  apply != 0 zeroes the residual
 * scale and codes of the others in place, which makes them contribute
 * exactly nothing to compensated attention.  Workspace: the per-vector keys. */
size_t bc_select_workspace_bytes(int n_slots, int64_t kv_stride);
int bc_select_residual_topk(bc_kv_planes P, int n_slots, int seq_len, int64_t kv_stride, int head_dim, int n_keep,
                            uint8_t* keep, int apply, void* workspace, size_t workspace_bytes, void* stream);

/* Staging of a decode step's host-resident inputs (no counterpart in the
 * reference): copies up to 4 segments (16-byte aligned, sizes multiples of 16)
 * from pinned host memory to device memory with one kernel launched with
 * programmatic dependent launch.  The kernel reads the sources before it waits
 * for the previous kernel in the stream (so the host-link latency overlaps
 * that kernel's tail; no earlier GPU work in the stream may write them) and
 * writes the destinations after it.  BitCache.step uses it for pinned Q, K, V:
 * every split CTA of the following bc_decode_step then reads its query from
 * device memory instead of crossing the host link (C3: 74 -> about 60 us). */
typedef struct bc_copy_seg {
    const void* src;
    void* dst;
    uint64_t bytes;
} bc_copy_seg;
int bc_stage_rows(const bc_copy_seg* segs, int n_segs, void* stream);

/* Log-sum-exp merge of n_parts partial triples per head (the cross-GPU sequence split):
 * parts[(p*n_heads + h)*(head_dim+2) + ...] as written by bc_decode_attention;
 * out fp16 [n_heads][head_dim]. */
int bc_lse_merge(const float* parts, int n_parts, int64_t n_heads, int head_dim, void* out, void* stream);

/* Head entropy over a plane cache's binary scores (same arithmetic as
 * bc_compute_head_entropy): entropy float [n_heads], query head h reads slot h. */
int bc_head_entropy_planes(const void* q, bc_kv_planes K, float* entropy, int n_heads, int seq_len,
                           int64_t kv_stride, int head_dim, void* stream);

/* XNOR popcount scores sum_w popc(~(q_w ^ k_w)) (xnor_dot.cuh:20-27) of each query head
 * against its slot's keys: out int32 [n_slots*group][seq_len]. */
int bc_xnor_popcount(const void* q, const void* k_sign, int32_t* out, int n_slots, int group, int seq_len,
                     int64_t kv_stride, int head_dim, void* stream);

/* Layout converters between reference records and planes (n vectors, flat). */
int bc_records_to_planes(const void* binvec, const void* resvec, bc_kv_planes out, int64_t n_vecs,
                         int head_dim, void* stream);
int bc_planes_to_records(bc_kv_planes in, void* binvec, void* resvec, int64_t n_vecs, int head_dim,
                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BITCACHE_B200_H */
