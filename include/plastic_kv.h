/*
 * plastic_kv.h — C ABI of the B200 (sm_100a) paged-KV decode hot path.
 *
 * The library (libplastic_kv.so) replaces three pure-PyTorch pieces of
 * plastic-infer's paged decode path:
 *   - the slot-mapping KV write        (src/plastic_infer/exec/runner_paged.py:112-129,
 *                                        src/plastic_infer/kv/kv_store.py:124-145)
 *   - paged GQA decode attention        (src/plastic_infer/exec/attention.py:103-190)
 *   - page moves between the device pool and the host chunk store
 *                                       (src/plastic_infer/kv/kv_store.py:230-334)
 *
 * Conventions
 *   - Plain pointers and sizes only; every device pointer is a CUDA device
 *     address owned by the caller (the library allocates nothing and keeps no
 *     pointer after a call returns).
 *   - Every function returns an int status: PI_OK (0) or a PI_ERR_* code.
 *     Arguments are validated on the host before any launch; a call that
 *     returns non-zero has launched nothing. (The reference's C entry point,
 *     src/plastic_infer/kernel/fast_index_copy.py:110-117, returns void.)
 *   - Kernels run on the caller's stream (`stream`, last argument), like the
 *     reference's ctypes launch on torch's current stream
 *     (src/plastic_infer/kernel/fast_index_copy.py:175-186).
 *   - `err` (optional, may be NULL) is a device int the kernels set to a
 *     PI_ERR_* code when they meet a bad index at run time (slot or page id out
 *     of range); the offending access is skipped, never faulted.
 *
 * Physical pool layout (the one thing that differs from the reference):
 *   K and V pools are each [num_pages, kv_heads, page_size, head_dim], i.e. the
 *   reference's logical [num_pages, kv_heads, head_dim, page_size]
 *   (src/plastic_infer/kv/kv_store.py:86-88) with the last two axes swapped in
 *   memory. A (page, kv-head) tile is one contiguous page_size*head_dim block and
 *   one token's row for one head is head_dim contiguous elements.
 */
#ifndef PLASTIC_KV_H_
#define PLASTIC_KV_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define PI_OK 0
#define PI_ERR_NULL_POINTER 1
#define PI_ERR_BAD_SHAPE 2
#define PI_ERR_MISALIGNED 3
#define PI_ERR_UNSUPPORTED 4
#define PI_ERR_CUDA 5
#define PI_ERR_WORKSPACE 6
#define PI_ERR_SLOT_RANGE 7   /* device-side: slot >= num_slots (write skipped)    */
#define PI_ERR_PAGE_RANGE 8   /* device-side: page id outside the pool (zero read)  */
#define PI_ERR_TIMEOUT 9      /* device-side: a bounded wait gave up                */
#define PI_ERR_SCRATCH_LIMIT 10 /* request needs more than the built-in scratch     */

/* element types */
#define PI_DTYPE_F32 0
#define PI_DTYPE_BF16 1
#define PI_DTYPE_F16 2

/* Version of this ABI (bumped on any signature change). */
int pi_abi_version(void);

/*
 * Programmatic dependent launch (no reference counterpart; off by default). When on,
 * the index-copy and the TMA attention kernels are launched with CUDA's programmatic
 * stream-serialization attribute. Each lets the next kernel on its stream launch as
 * soon as it has started. The index-copy waits for the previous kernel before reading
 * anything. The attention kernel reads only `ctx_lens` and `block_tables` before
 * waiting: it computes its work split and fetches its first page ids while the
 * previous kernel (e.g. the step's index-copy) finishes.
 *
 * So with it on, `ctx_lens` and `block_tables` must not be written by the kernel
 * launched immediately before the attention on the same stream (host copies are
 * fine). Applies to launches made after the call, in every thread. Returns PI_OK.
 */
int pi_set_programmatic_launch(int enable);

/*
 * Page-ring depth of plain pi_paged_decode_attn launches (no reference counterpart).
 * The TMA kernel keeps a ring of page stages per warp. By default (AUTO) a launch
 * whose bound on the work (batch x bt_stride x num_kv_heads x num_q_heads /
 * num_kv_heads) is large uses a two-stage ring with two CTAs per SM, and every other
 * launch a deep ring (4 stages at head_dim <= 128) with one CTA per SM. DEEP and SHALLOW force one of the
 * two for every plain launch the fast path takes (SHALLOW only where two CTAs fit on
 * an SM), so either instance can be run and checked at any size. Results agree
 * within the attention tolerance; they are not bit-identical because the work split
 * differs. Launches with the fused append or the peer all-gather always use the deep
 * ring. Applies to launches made after the call, in every thread. Returns PI_OK, or
 * PI_ERR_BAD_SHAPE for an unknown mode.
 */
#define PI_ATTN_RING_AUTO 0
#define PI_ATTN_RING_DEEP 1
#define PI_ATTN_RING_SHALLOW 2
int pi_set_decode_attn_ring(int mode);

/* Static description of a status code. Never NULL. */
const char* pi_error_string(int code);

/*
 * Slot-mapping KV write: for i in [0, n_tokens) with s = slot_mapping[i] >= 0,
 *   k_pool[s / page_size, h, s % page_size, :] = k_new[i, h, :]   (all h)
 *   v_pool[...]                                = v_new[i, h, :]
 * A negative slot is padding and is skipped. Bit-exact element copy.
 *
 * Duplicate slots: when two tokens of one launch name the same non-negative slot,
 * every 16-byte piece of that slot's rows ends up holding the bytes of one of them,
 * but which one is unspecified (and may differ from piece to piece). The
 * reference's per-token loop keeps the last token's row; a caller that relies on
 * that must not pass duplicates in one launch (split the batch, or drop all but the
 * last occurrence). Slots that differ never interfere.
 *
 * Replaces the per-token Python loop of _write_kv_layer
 * (src/plastic_infer/exec/runner_paged.py:123-129) and the per-layer write of
 * KVRequestCache.append_token (src/plastic_infer/kv/kv_store.py:140-143); slot
 * addressing follows BlockTable.get_page (src/plastic_infer/kv/paged.py:54-59):
 * slot = page_id * page_size + offset.
 *
 *   k_new, v_new   [n_tokens, kv_heads, head_dim] with token stride
 *                  `src_token_stride` elements (heads are contiguous rows)
 *   slot_mapping   [n_tokens] int64, device
 *   num_slots      num_pages * page_size (bound for slots)
 */
int pi_kv_index_copy(void* k_pool, void* v_pool, const void* k_new, const void* v_new,
                     const int64_t* slot_mapping, int64_t n_tokens, int kv_heads, int head_dim,
                     int page_size, int64_t num_slots, int dtype, int64_t src_token_stride,
                     int* err, cudaStream_t stream);

/*
 * Bytes of device workspace pi_paged_decode_attn needs for this shape on the
 * current device (it depends on head_dim and the SM count only). The first
 * pi_paged_decode_attn_ws_zero_bytes() bytes hold arrival counters at a fixed
 * place for every shape: they must be zero before the first call and every
 * completed call leaves them zero again, so one zero-fill when the workspace is
 * allocated suffices. After a call that reported PI_ERR_TIMEOUT through `err`,
 * zero them again. Calls sharing one workspace must be ordered (one stream).
 */
size_t pi_paged_decode_attn_workspace_bytes(int batch, int num_q_heads, int num_kv_heads,
                                            int head_dim);
size_t pi_paged_decode_attn_ws_zero_bytes(void);

/*
 * Page-ring stages a plain pi_paged_decode_attn launch of this shape would use on
 * the current device under the current pi_set_decode_attn_ring mode (no reference
 * counterpart): 2 for the shallow ring with two CTAs per SM, the deep ring's depth
 * otherwise, or 0 when the shape takes the generic SIMT path. Pointer alignment is
 * not considered (misaligned pools or q also send a launch to the SIMT path).
 */
int pi_paged_decode_attn_ring_stages(int batch, int64_t bt_stride, int num_q_heads,
                                     int num_kv_heads, int head_dim, int page_size,
                                     int64_t num_pages, int dtype);

/*
 * Batched paged GQA decode attention, one query token per request:
 *   out[b, hq, :] = softmax(scale * q[b, hq, :] . K_b[hq / G]^T) V_b[hq / G]
 * over the first ctx_lens[b] tokens of request b, whose pages are
 * block_tables[b, 0 .. ceil(ctx_lens[b] / page_size)), G = num_q_heads / num_kv_heads.
 * fp32 softmax and accumulation; a request with ctx_lens[b] == 0 gets zeros.
 *
 * Replaces gather_paged_kv + repeat_interleave + scaled_dot_product_attention of
 * paged_attention_v1 (src/plastic_infer/exec/attention.py:103-190) for Sq == 1,
 * batched over requests (the reference calls it once per request through
 * _attn_paged, src/plastic_infer/exec/runner_paged.py:36-59). GQA mapping
 * hq -> hq // G as at attention.py:183-187; default scale 1/sqrt(head_dim) as SDPA.
 *
 *   q, out         [batch, num_q_heads, head_dim], row stride q_stride / out_stride
 *                  elements between consecutive requests (dtype of the pools)
 *   block_tables   [batch, bt_stride] int32 page ids, device
 *   ctx_lens       [batch] int32, device
 *   workspace      >= pi_paged_decode_attn_workspace_bytes(...) bytes, 256-B aligned
 */
int pi_paged_decode_attn(void* out, const void* q, const void* k_pool, const void* v_pool,
                         const int32_t* block_tables, int64_t bt_stride, const int32_t* ctx_lens,
                         int batch, int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                         int64_t num_pages, float scale, int dtype, int64_t q_stride,
                         int64_t out_stride, void* workspace, size_t workspace_bytes, int* err,
                         cudaStream_t stream);

/*
 * Decode step of one layer in one launch: the slot-mapping write of the step's new
 * K/V rows followed by paged decode attention. Same result as
 *   pi_kv_index_copy(k_pool, v_pool, k_new, v_new, slot_mapping, batch, ...)
 *   pi_paged_decode_attn(out, q, k_pool, v_pool, ...)
 * with one new row per request (k_new, v_new: [batch, kv_heads, head_dim], request
 * stride new_stride elements; slot_mapping[b] < 0 = no new row for request b).
 * The page holding request b's new slot must be read only by request b (the
 * reference never shares pages between requests, src/plastic_infer/kv/paged.py:12).
 * Replaces the per-layer pair _write_kv_layer + _attn_paged of the decode loop
 * (src/plastic_infer/exec/runner_paged.py:250-255). Shapes the fused kernel does
 * not cover run the two kernels back to back.
 */
int pi_paged_decode_attn_append(void* out, const void* q, void* k_pool, void* v_pool,
                                const void* k_new, const void* v_new,
                                const int64_t* slot_mapping, int64_t new_stride,
                                const int32_t* block_tables, int64_t bt_stride,
                                const int32_t* ctx_lens, int batch, int num_q_heads,
                                int num_kv_heads, int head_dim, int page_size, int64_t num_pages,
                                float scale, int dtype, int64_t q_stride, int64_t out_stride,
                                void* workspace, size_t workspace_bytes, int* err,
                                cudaStream_t stream);

/*
 * Multi-GPU decode attention with the all-gather fused into the kernel (no
 * counterpart in the reference, which runs on one GPU; the exchange point is where
 * the attention output meets o_proj, src/plastic_infer/exec/runner_paged.py:256-258).
 *
 * Each of `world` ranks holds the KV heads of one head shard and attends its own
 * query heads (as pi_paged_decode_attn). Every rank owns a gathered-output buffer
 * [world][batch][num_q_heads_local][head_dim] that all ranks have mapped (CUDA IPC);
 * a rank writes its own slice of EVERY rank's buffer with NVLink peer stores as soon
 * as each (request, KV head) row group is final. When all of a launch's stores have
 * landed, the launch writes `epoch` into peer_flags[r][rank] on every rank r, then
 * waits (bounded, ~2 s; PI_ERR_TIMEOUT through `err` on expiry) until its own
 * flags[r] >= epoch for all r. When the launch completes, the whole gathered buffer
 * is in place for the work that follows it on `stream` (o_proj). Epochs increase by
 * one per launch on every rank.
 *
 *   out           must be peer_out[rank] + rank * rank_stride (this rank's slice of its
 *                 own gathered buffer); out_stride as for pi_paged_decode_attn
 *   workspace     as for pi_paged_decode_attn (its zeroed block also holds the
 *                 launch-completion counter)
 * Peer pointers are device addresses valid in this process (cudaIpcOpenMemHandle).
 * Plain peer stores and flag writes only: no TMA or multicast access to peer memory.
 *
 * Output slots: consecutive launches must write different buffers (peer_out), so that
 * a rank's stores for launch e never land in a buffer a peer still reads for launch
 * e - 1; two buffers used alternately are enough, because launch e on any rank starts
 * only after every rank has finished launch e - 1's work and hence the reads of
 * launch e - 2's output that preceded it in stream order.
 *
 * Epochs from the device: with launch_counter != NULL (a word in this rank's own
 * memory counting its completed gather launches, zero at start) `epoch` is ignored;
 * a launch uses *launch_counter + 1 and stores it back. The arguments of every
 * launch are then the same from step to step, so a sequence of launches can be
 * captured in a CUDA graph and replayed (a sequence whose length is a multiple of the
 * number of output slots keeps the alternation across replays).
 */
#define PI_MAX_PEERS 8
typedef struct pi_peer_gather {
  void* peer_out[PI_MAX_PEERS];
  unsigned* peer_flags[PI_MAX_PEERS];
  int rank;
  int world;
  int64_t rank_stride;
  unsigned epoch;
  unsigned* launch_counter;
} pi_peer_gather_t;

int pi_paged_decode_attn_gather(void* out, const void* q, const void* k_pool, const void* v_pool,
                                const int32_t* block_tables, int64_t bt_stride,
                                const int32_t* ctx_lens, int batch, int num_q_heads,
                                int num_kv_heads, int head_dim, int page_size, int64_t num_pages,
                                float scale, int dtype, int64_t q_stride, int64_t out_stride,
                                void* workspace, size_t workspace_bytes,
                                const pi_peer_gather_t* gather, int* err, cudaStream_t stream);

/*
 * Allocation-free pi_paged_decode_attn (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory when they attend: a host loop
 * that reaches this library only through this C ABI and owns no CUDA allocator,
 * or an engine whose memory planner has already given every free byte to the
 * page pool and the weights, so that a cudaMalloc during decoding would fail or
 * stall the device. Same arguments and results as pi_paged_decode_attn, minus the
 * workspace: the split-KV scratch is one array of PI_NOALLOC_SCRATCH_BYTES
 * compiled into the library, which every GPU that loads the library holds until
 * the process exits. The function calls no cudaMalloc / cudaFree and no
 * allocating library routine.
 *
 *   - A request that takes the TMA fast path and whose scratch need
 *     (pi_paged_decode_attn_workspace_bytes) exceeds PI_NOALLOC_SCRATCH_BYTES is
 *     rejected with PI_ERR_SCRATCH_LIMIT before any launch (e.g. head_dim 256, or
 *     head_dim 128 on a GPU with more than 148 SMs). Shapes served by the generic
 *     SIMT path (fp32 pools, other head_dim or page sizes, G > 8) use no scratch and
 *     are never rejected for it.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current and caches it; make that
 *     first call before any stream capture on the device.
 *   - All calls share the one array and it keeps the last call's contents; each
 *     call clears the part that must start at zero (a cudaMemsetAsync on `stream`).
 *     Calls that overlap on the GPU (other streams, other threads) race on it:
 *     order them on one stream.
 */
#define PI_NOALLOC_SCRATCH_BYTES ((size_t)12 << 20)
int pi_paged_decode_attn_noalloc(void* out, const void* q, const void* k_pool,
                                 const void* v_pool, const int32_t* block_tables,
                                 int64_t bt_stride, const int32_t* ctx_lens, int batch,
                                 int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                 int64_t num_pages, float scale, int dtype, int64_t q_stride,
                                 int64_t out_stride, int* err, cudaStream_t stream);

/*
 * Paged prefill attention of one request: q_len new tokens against the first kv_len
 * tokens of its pages, straight from the pool (replaces the prefill branch of
 * _attn_paged, src/plastic_infer/exec/runner_paged.py:36-95: gather_paged_kv +
 * repeat_interleave + SDPA, with is_causal when q_start_pos == 0 and a dense mask
 * otherwise).
 *   out[i, h, :] = softmax(scale * q[i, h, :] . K_{h/G}[j]) V_{h/G}[j]   over
 *   j < lim(i),  lim(i) = min(kv_len, q_start + i + 1) if causal, else kv_len.
 * With q_start == 0 and causal this is SDPA's is_causal (top-left aligned); with
 * q_start > 0 it is the reference's offset mask (query i at position q_start + i).
 *   q, out        [q_len, num_q_heads, head_dim], token strides q_tok_stride /
 *                 out_tok_stride elements (heads contiguous)
 *   block_table   [table_len] int32 page ids, device; kv_len <= table_len * page_size
 * bf16 or f16 pools; head_dim 64 or 128; page_size 16 or 32; num_q_heads / num_kv_heads
 * in {1, 2, 4, 8, 16}. Other shapes return PI_ERR_UNSUPPORTED. fp32 softmax and
 * accumulation. Rows with no key (kv_len == 0) are zero.
 */
int pi_paged_prefill_attn(void* out, const void* q, const void* k_pool, const void* v_pool,
                          const int32_t* block_table, int64_t table_len, int q_len, int kv_len,
                          int q_start, int causal, int num_q_heads, int num_kv_heads,
                          int head_dim, int page_size, int64_t num_pages, float scale, int dtype,
                          int64_t q_tok_stride, int64_t out_tok_stride, int* err,
                          cudaStream_t stream);

/*
 * pi_paged_prefill_attn on the 5th-generation tensor cores (tcgen05): same arguments,
 * semantics, shape coverage and errors, plus q and out must be 16-byte aligned with
 * q_tok_stride and out_tok_stride multiples of 8 elements (PI_ERR_MISALIGNED otherwise):
 * both move by TMA. A CTA takes 128 query rows of one KV head; S = Q K^T and O = P V
 * accumulate in tensor memory, K/V pages stream through a TMA ring, every wait is bounded
 * (PI_ERR_TIMEOUT through `err`). Only the q_len x num_q_heads x head_dim output rows are
 * written.
 * Same replaced reference code as pi_paged_prefill_attn
 * (src/plastic_infer/exec/runner_paged.py:36-95).
 */
int pi_paged_prefill_attn_tc(void* out, const void* q, const void* k_pool, const void* v_pool,
                             const int32_t* block_table, int64_t table_len, int q_len,
                             int kv_len, int q_start, int causal, int num_q_heads,
                             int num_kv_heads, int head_dim, int page_size, int64_t num_pages,
                             float scale, int dtype, int64_t q_tok_stride,
                             int64_t out_tok_stride, int* err, cudaStream_t stream);

/*
 * One span of a KV sequence for pi_host_stream_attn: `len` tokens whose K element
 * (kv head h, token t, dim d) is k[h * head_stride + t * tok_stride + d * dim_stride]
 * (V the same with v). k and v point to device memory or to page-locked host memory
 * (cudaHostAlloc / cudaHostRegister), which the kernel reads in place through its
 * mapped device alias. Strides are in elements and non-negative.
 */
typedef struct pi_kv_span {
  const void* k;
  const void* v;
  int64_t len;
  int64_t head_stride;
  int64_t tok_stride;
  int64_t dim_stride;
} pi_kv_span_t;

#define PI_HS_MAX_SPANS 512

/*
 * Attention of one request over a KV sequence split into spans (replaces
 * host_stream_attention_v1, src/plastic_infer/exec/attention.py:193-250: host chunks
 * [H_kv, D, C] oldest first, then the resident tail [1, R, H_kv, D], concatenated,
 * GQA-expanded and fed to SDPA). The spans are concatenated in order into positions
 * [0, kv_len); host spans cross the host link once and are never staged.
 *   out[i, h, :] = softmax_j(scale * q[i, h, :] . K_{h/G}[j]) V_{h/G}[j]
 * over every j when causal == 0, else over j <= q_start + i (the reference's offset
 * mask; with q_start == 0 and q_len == kv_len this is SDPA's is_causal). Rows with no
 * visible key are zero.
 *   q, out   device, [q_len, num_q_heads, head_dim], token strides q_tok_stride /
 *            out_tok_stride elements, heads and dims contiguous
 *   spans    HOST array of num_spans <= PI_HS_MAX_SPANS descriptors, read during the
 *            call; a span whose memory has no device alias (pageable host memory)
 *            returns PI_ERR_UNSUPPORTED
 *   workspace  device scratch of pi_host_stream_attn_workspace_size(...) bytes,
 *            256-byte aligned (none needed when that size is 0)
 *   flags    0, or PI_HS_SPANS_CHECKED: the caller has established that every span
 *            is device memory or page-locked host memory, and the library then skips
 *            its per-span pointer queries (about a microsecond each) and uses host
 *            addresses as device addresses, as unified addressing maps pinned memory
 *            (registered memory only where the device reports it can use host pointers)
 * dtype f32, bf16 or f16 for q, out and every span; head_dim a multiple of 8, <= 256;
 * fp32 arithmetic. Two launches (splits, then their merge) when the sequence is long
 * enough to be split, else one.
 */
size_t pi_host_stream_attn_workspace_size(int q_len, int num_q_heads, int num_kv_heads,
                                          int head_dim, int64_t kv_len);
#define PI_HS_SPANS_CHECKED 1
int pi_host_stream_attn(void* out, const void* q, int64_t q_tok_stride, int64_t out_tok_stride,
                        const pi_kv_span_t* spans, int num_spans, int q_len, int64_t q_start,
                        int causal, int num_q_heads, int num_kv_heads, int head_dim, float scale,
                        int dtype, void* workspace, size_t workspace_bytes, int flags, int* err,
                        cudaStream_t stream);

/*
 * MoE expert-slot copy, all banks in one launch (replaces the reference's fused
 * multi-bank copy, plasticinfer_fast_index_copy_multi_launch:
 * src/plastic_infer/kernel/fast_index_copy.py:190-244, kernel
 * src/plastic_infer/kernel/csrc/jit/fast_index_copy.cuh:436-503; called by
 * OffloadMoeCache.copy_missing, src/plastic_infer/moe/offload_cache.py:998-1012). Same
 * arguments and meaning:
 *   for b < num_banks, i < n:  dst_b[dst_indices[i]] = src_b[src_indices[i]]
 * with row bytes feat_bytes[b], base addresses dst_ptrs[b] / src_ptrs[b] (int64 device
 * arrays; the sources are pinned host banks read through their device alias), and
 * n = min(num_indices[0], length) when num_indices (device int64 [1]) is given, else
 * length. Indices are int32 when use_int32 != 0, else int64. A bank whose row bytes or
 * base addresses are not 16-byte multiples is skipped with PI_ERR_MISALIGNED in `err`; a
 * negative index skips its row with PI_ERR_SLOT_RANGE. Destination rows must be distinct.
 * At most 32 banks.
 */
int pi_expert_slot_copy(const int64_t* dst_ptrs, const int64_t* src_ptrs,
                        const int64_t* feat_bytes, int num_banks, const void* dst_indices,
                        const void* src_indices, int64_t length, const int64_t* num_indices,
                        int use_int32, int* err, cudaStream_t stream);

/*
 * Fused decode prologue of one layer (no single reference counterpart; it replaces the
 * op sequence qk_norm -> rope_positions on q and k -> _write_kv_layer of the reference
 * runners: src/plastic_infer/exec/attention.py:23-95 and
 * src/plastic_infer/exec/runner_paged.py:112-129, runner_moe_paged.py:135-142). For each
 * request b (one new token at position positions[b]):
 *   q_out[b, h]   = rope(qknorm(q_in[b, h], q_norm_w), positions[b])      h < Hq
 *   K slot[b], h  = rope(qknorm(k_in[b, h], k_norm_w), positions[b])      h < Hkv
 *   V slot[b], h  = v_in[b, h]
 * qknorm(x, w) = x / sqrt(mean(x^2) + eps) * w over head_dim (skipped when both weights
 * are NULL); rope is rotate_half with angle positions[b] * inv_freq[j mod D/2] in fp32
 * (inv_freq [head_dim/2] fp32 on the device, e.g. 1 / base^(2j/D) as build_rope_cache
 * computes it). fp32 arithmetic, one rounding to the pool dtype. slot_mapping[b] < 0
 * writes no K/V row for b; the pools are the physical [P, Hkv, S, D] layout.
 *   q_in, k_in, v_in   projection outputs in `in_dtype`; request strides q_in_stride
 *                      and kv_in_stride elements (heads contiguous): separate q/k/v
 *                      tensors or the three slices of one fused QKV output
 *   q_out              pool dtype, request stride q_out_stride elements
 * head_dim 64, 128 or 256.
 */
int pi_decode_prologue(void* q_out, int64_t q_out_stride, void* k_pool, void* v_pool,
                       const void* q_in, int64_t q_in_stride, const void* k_in, const void* v_in,
                       int64_t kv_in_stride, int in_dtype, const void* q_norm_w,
                       const void* k_norm_w, float eps, const float* inv_freq,
                       const int64_t* positions, const int64_t* slot_mapping, int batch,
                       int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                       int64_t num_slots, int pool_dtype, int* err, cudaStream_t stream);

/*
 * Contiguous gather of a request's pages in the reference's gather layout:
 *   out[t, h, :] = pool[block_table[t / page_size], h, t % page_size, :]
 * for t in [0, num_tokens). out is [num_tokens, kv_heads, head_dim].
 * Replaces gather_paged_kv's index_select + permute + reshape
 * (src/plastic_infer/exec/attention.py:133-148) for one pool.
 */
int pi_paged_kv_gather(void* out, const void* pool, const int32_t* block_table, int64_t num_tokens,
                       int kv_heads, int head_dim, int page_size, int64_t num_pages, int dtype,
                       int* err, cudaStream_t stream);

/*
 * Page gather (pool -> contiguous staging) and scatter (staging -> pool).
 * Page i of the list (page id page_ids[i]) holds kv_heads tiles of `tile_bytes`
 * bytes (tile_bytes = page_size * head_dim * elem). In the staging buffer, pages
 * are grouped `pages_per_group` at a time and laid out head-major inside a group:
 *   staging offset of (page i, head h) =
 *       ((i / ppg) * kv_heads + h) * ppg * tile_bytes + (i % ppg) * tile_bytes
 * With ppg = pages_per_chunk and groups = layers this is the host chunk layout
 * [n_layers, kv_heads, tokens_per_chunk, head_dim], i.e. the reference's chunk
 * [n_layers, kv_heads, head_dim, tokens_per_chunk]
 * (src/plastic_infer/kv/kv_store.py:252-269) with its last two axes swapped.
 * With ppg = 1 pages are simply concatenated.
 * Replaces the per-page .to("cpu") / .to(device) loops of
 * KVStore.sink_completed_chunks (src/plastic_infer/kv/kv_store.py:258-269) and
 * KVStore.load_prefix (src/plastic_infer/kv/kv_store.py:311-321); the host<->device
 * leg is one cudaMemcpyAsync of the staging buffer issued by the caller.
 * Page ids outside [0, num_pages) are skipped and reported through `err`.
 */
int pi_page_gather(void* staging, const void* pool, const int32_t* page_ids, int64_t n_pages,
                   int kv_heads, int64_t tile_bytes, int pages_per_group, int64_t num_pages,
                   int* err, cudaStream_t stream);
int pi_page_scatter(void* pool, const void* staging, const int32_t* page_ids, int64_t n_pages,
                    int kv_heads, int64_t tile_bytes, int pages_per_group, int64_t num_pages,
                    int* err, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PLASTIC_KV_H_ */
