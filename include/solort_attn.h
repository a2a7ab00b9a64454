/*
 * solort_attn.h -- C ABI of the B200 (sm_100a) grouped-query attention engine for SoloRT's Qwen3
 * fast path.
 *
 * Every entry point takes raw device pointers, element strides and sizes; no torch types cross
 * this boundary. All kernels are enqueued on the caller's stream (a cudaStream_t passed as
 * `void*`), never allocate (only the set-up calls solort_attn_exchange_buffer_create / _open map
 * memory), never synchronise the host, and read lengths / positions from device memory, so every
 * per-step call can be captured inside a CUDA graph. Return value: SOLORT_OK (0) or a
 * negative SOLORT_ERR_* code; no exception crosses the ABI and nothing falls back to another
 * implementation.
 *
 * State the library keeps: on the host, per-device properties, one-time kernel attribute set-up
 * and a small cache of encoded K/V tensor maps keyed by every input of the encoding (a hit is the
 * descriptor a fresh encoding would give, so freed and reused buffers are harmless); on each
 * device, the status flags read by solort_attn_device_status and the static scratch array of
 * solort_attn_decode_static_scratch. Calls from several host threads are safe.
 *
 * The reference (owen920831/SoloRT) computes this attention inline in torch; the entry points
 * replace these call sites (paths inside the reference project):
 *   solort_attn_decode, q_len == 1, static KV:
 *       src/solort/model/cuda_graph_executor.py:168,180-184   (grouped decode + live-length mask)
 *   solort_attn_decode, q_len == K+1, static KV:
 *       src/solort/model/cuda_graph_executor.py:250,261-263   (verify: masked SDPA over max_len)
 *   solort_attn_decode with a block table (paged KV, NHD pages [pages, 2, P, nkv, hd]):
 *       src/solort/backends/transformers_flashinfer.py:95-129  (AttentionInterface decode/prefill)
 *       src/solort/cache/kv_cache.py:86-100,136-149            (page layout, slot = bt[p//P]*P+p%P)
 *   solort_attn_kv_store (slot-mapped K/V mirror into the paged arena):
 *       src/solort/cache/kv_cache.py:191-235, called from transformers_flashinfer.py:93,205-220
 *   solort_attn_decode with out_f32/lse_out + solort_attn_lse_merge, and
 *   solort_attn_decode_exchange + solort_attn_exchange_merge:
 *       no counterpart (the reference is single-GPU); sequence-sharded long-context decode.
 */
#ifndef SOLORT_ATTN_H_
#define SOLORT_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SOLORT_ATTN_ABI_VERSION 3

#if defined(__GNUC__)
#define SOLORT_API __attribute__((visibility("default")))
#else
#define SOLORT_API
#endif

/* Status codes. */
#define SOLORT_OK 0
#define SOLORT_ERR_INVALID_ARGUMENT (-1) /* null pointer, bad size, misaligned pointer/stride */
#define SOLORT_ERR_UNSUPPORTED (-2)      /* head_dim != 128, too many query rows per KV head */
#define SOLORT_ERR_WORKSPACE (-3)        /* workspace missing or smaller than required */
#define SOLORT_ERR_CUDA (-4)             /* a CUDA runtime call or kernel launch failed */
#define SOLORT_ERR_TENSOR_MAP (-5)       /* the driver rejected a TMA descriptor */
#define SOLORT_ERR_NO_DEVICE (-6)        /* no sm_100 device is current */
#define SOLORT_ERR_SCRATCH_LIMIT (-7)    /* the call needs more split scratch than the static 4 MiB */
#define SOLORT_ERR_IPC (-8)              /* a CUDA IPC export / import of an exchange buffer failed */

/*
 * GQA attention of q_len query tokens per sequence against a KV cache: decode (q_len == 1),
 * speculative verify / chunked append (q_len > 1), static buffer or paged.
 *
 * Shapes (element strides; head_dim must be 128 and contiguous):
 *   q    [batch, q_len, num_qo_heads, head_dim] bf16
 *   out  [batch, q_len, num_qo_heads, head_dim] bf16
 *   K, V static  : element (token t, kv head h, dim d) at k + t*kv_stride_token
 *                  + h*kv_stride_head + d  (NHD [max_len, nkv, hd] or HND [nkv, max_len, hd])
 *   K, V paged   : element (page p, row r, head h, dim d) at k + p*kv_stride_page
 *                  + r*kv_stride_token + h*kv_stride_head + d; V likewise from v. For SoloRT's
 *                  NHD arena [pages, 2, P, nkv, hd]: v = k + P*nkv*hd, kv_stride_page = 2*P*nkv*hd.
 *   block_table  [batch, >= ceil(kv_len/P)] int32 physical page ids (NULL for a static cache)
 *
 * Positions (read on the device, so the call can sit in a graph whose position changes):
 *   q_pos[b] (int64) is the absolute position of query row 0 of sequence b; query row i sits at
 *   q_pos[b] + i and attends key position j iff j <= q_pos[b] + i. Local key t of this cache sits
 *   at position kv_pos_offset + t (0 unless the cache is one shard of a longer sequence).
 *   q_lens (int32 [batch], optional) gives a per-sequence query count <= q_len; rows past it are
 *   neither computed nor written.
 *   max_kv_len is a host-side upper bound on the number of local keys any row sees; it sizes the
 *   grid (the reference's decode bucket `bound`). Keys past it are not read.
 *
 * Outputs: by default bf16 `out`. If lse_out != NULL the call instead writes the normalised fp32
 * output to out_f32 [batch, q_len, num_qo_heads, head_dim] (contiguous) and the natural-log
 * log-sum-exp of the scaled scores to lse_out [batch, q_len, num_qo_heads]; rows that see no key
 * get out_f32 = 0, lse = -inf. These partials combine with solort_attn_lse_merge.
 *
 * Workspace: split-KV partials; query solort_attn_decode_workspace_size() with the same args.
 *
 * flags: SOLORT_DECODE_STABLE_PREFIX promises that q_pos, q_lens, the block table and every K/V
 * row at a position below q_pos[b] were written before the kernel launched just before this call
 * on the stream (earlier steps, host copies before a graph replay), so the call may read them
 * while that kernel is still running: the key stream then starts during its tail. Rows at q_pos[b]
 * and later (the tokens the previous kernel may just have appended), the queries and the
 * workspace are touched only after it has finished, with or without the flag.
 */
#define SOLORT_DECODE_STABLE_PREFIX 1u
typedef struct SolortDecodeArgs {
  const void* q;
  int64_t q_stride_batch, q_stride_token, q_stride_head;
  void* out;
  int64_t out_stride_batch, out_stride_token, out_stride_head;
  float* out_f32;
  float* lse_out;

  const void* k;
  const void* v;
  int64_t kv_stride_token, kv_stride_head, kv_stride_page;
  int32_t kv_capacity; /* static: tokens in the buffer. paged: ignored */

  const int32_t* block_table;
  int64_t block_table_stride;
  int32_t page_size; /* power of two >= 8 */
  int32_t num_pages; /* physical pages in the arena */

  const int64_t* q_pos;
  const int32_t* q_lens;
  int64_t kv_pos_offset;

  int32_t batch, q_len, num_qo_heads, num_kv_heads, head_dim;
  int32_t max_kv_len;
  float scale;
  int32_t num_splits; /* 0 = choose for the device; otherwise the number of key splits */

  void* workspace;
  size_t workspace_bytes;
  uint32_t flags; /* SOLORT_DECODE_* bits, 0 by default */
} SolortDecodeArgs;

SOLORT_API int solort_attn_decode_workspace_size(const SolortDecodeArgs* args, size_t* bytes);
SOLORT_API int solort_attn_decode(const SolortDecodeArgs* args, void* stream);

/*
 * solort_attn_decode for callers that cannot allocate device memory. It has no counterpart in the
 * reference. Some callers have no way to provide a workspace: a plugin host whose operator
 * interface passes only input and output buffers, or a host runtime that binds this C ABI but has
 * no CUDA allocator of its own. This entry point takes the same arguments, ignores `workspace` /
 * `workspace_bytes`, and keeps the split partials in a 4 MiB device array inside the library
 * instead; it calls no allocator.
 *
 *  - Limit: calls whose split partials need more than 4 MiB (solort_attn_decode_workspace_size)
 *    are rejected with SOLORT_ERR_SCRATCH_LIMIT; use solort_attn_decode with a workspace for them.
 *    Decode of one sequence with 32 query heads (37 splits) needs about 0.6 MiB.
 *  - The array exists on a GPU from the moment the library's device code is loaded in that GPU's
 *    context (at the latest, the first call on it) until that context is destroyed.
 *  - Each call looks up the array's device address on the current device. The first call in a
 *    device context loads the device code, which a stream capture does not allow: make that first
 *    call before any stream capture on that device.
 *  - All calls on a GPU share the array and it keeps the last call's contents. Nothing in it needs
 *    to start at zero (a call writes every part it reads), but calls that overlap on the GPU, for
 *    example on two streams, race on it: serialise them.
 */
SOLORT_API int solort_attn_decode_static_scratch(const SolortDecodeArgs* args, void* stream);

/*
 * Merge num_parts partial results over disjoint key sets into one:
 *   O = sum_p exp(lse_p - lse*) O_p / sum_p exp(lse_p - lse*),  lse = lse* + log(sum_p ...).
 * o_parts: part p, row r at o_parts + p*part_stride + r*head_dim (fp32, head_dim contiguous);
 * lse_parts: part p, row r at lse_parts + p*lse_part_stride + r.
 * Rows are (batch, token, head) flattened, rows = batch*q_len*num_qo_heads. Writes bf16 `out`
 * (strided like SolortDecodeArgs.out) unless out_f32 != NULL, in which case it writes fp32
 * out_f32[r*head_dim + d] and lse_out[r].
 */
typedef struct SolortMergeArgs {
  const float* o_parts;
  int64_t part_stride;
  const float* lse_parts;
  int64_t lse_part_stride;
  int32_t num_parts;
  int32_t batch, q_len, num_qo_heads, head_dim;
  void* out;
  int64_t out_stride_batch, out_stride_token, out_stride_head;
  float* out_f32;
  float* lse_out;
} SolortMergeArgs;

SOLORT_API int solort_attn_lse_merge(const SolortMergeArgs* args, void* stream);

/*
 * Sequence-sharded decode with a peer-memory exchange. No counterpart in the reference (it runs on
 * one GPU); this replaces the all-gather + merge of a partial per rank with direct NVLink stores.
 *
 * Each of R ranks (one process per GPU, R <= SOLORT_MAX_RANKS) holds a contiguous shard of the
 * keys. solort_attn_decode_exchange runs the split-KV decode over the local shard (args as for
 * solort_attn_decode; out, out_f32, lse_out and q_lens must be NULL) and its merge kernel stores
 * the rank's partial into slot_in_rank[p] on every rank p -- this rank's slot in p's receive
 * buffer, a peer pointer for p != rank. A slot is rows*129 64-bit words (rows =
 * batch*q_len*num_qo_heads): word r*128+d holds O[r][d], word rows*128+r the natural-log LSE of
 * row r, each as (1 << 32) | float bits, written with one 64-bit store, so every word carries its
 * own arrival mark and no fence or flag is needed. solort_attn_exchange_merge, on every rank,
 * waits until all R slots of each row are marked (one second at most per row; on expiry it sets
 * bit 3 of the device status and leaves the row unwritten), merges the R partials into bf16
 * `out` and zeroes the words it read, ready for the next use of the slots.
 *
 * Slots live in buffers from solort_attn_exchange_buffer_create (cudaMalloc'd, zero-filled,
 * exported as a CUDA IPC handle) and solort_attn_exchange_buffer_open (the peer mapping). A set of
 * slots may be reused by a later call once every rank has finished the exchange_merge that read
 * it -- for example one set per layer of a decode step. Workspace: query
 * solort_attn_decode_exchange_workspace_size() with the same args.
 */
#define SOLORT_MAX_RANKS 8
typedef struct SolortExchangeArgs {
  int32_t num_ranks;
  int32_t rank;
  uint64_t* slot_in_rank[SOLORT_MAX_RANKS]; /* rows*129 words in rank p's memory, 16-aligned */
} SolortExchangeArgs;

SOLORT_API int solort_attn_decode_exchange_workspace_size(const SolortDecodeArgs* args,
                                                          size_t* bytes);
SOLORT_API int solort_attn_decode_exchange(const SolortDecodeArgs* args,
                                           const SolortExchangeArgs* exchange, void* stream);

typedef struct SolortExchangeMergeArgs {
  uint64_t* slots;     /* rank s's slot (rows*129 words) at slots + s*slot_stride */
  int64_t slot_stride; /* words between consecutive ranks' slots (>= rows*129, even) */
  int32_t num_ranks;
  int32_t batch, q_len, num_qo_heads, head_dim;
  void* out; /* bf16, strided like SolortDecodeArgs.out */
  int64_t out_stride_batch, out_stride_token, out_stride_head;
} SolortExchangeMergeArgs;

SOLORT_API int solort_attn_exchange_merge(const SolortExchangeMergeArgs* args, void* stream);

/* Exchange buffers (set-up calls, not for the per-step path): create allocates `bytes` of device
 * memory on the current device, zero-fills it and writes its 64-byte CUDA IPC handle; open maps a
 * peer's buffer from its handle; close unmaps an opened buffer; destroy frees a created one. */
SOLORT_API int solort_attn_exchange_buffer_create(size_t bytes, void** ptr, void* ipc_handle);
SOLORT_API int solort_attn_exchange_buffer_open(const void* ipc_handle, void** ptr);
SOLORT_API int solort_attn_exchange_buffer_close(void* ptr);
SOLORT_API int solort_attn_exchange_buffer_destroy(void* ptr);

/*
 * Causal (or full) GQA prefill on the tcgen05 tensor cores, one sequence.
 *   q   [q_len,  num_qo_heads, 128] bf16, element strides (q_stride_token, q_stride_head)
 *   k,v [kv_len, num_kv_heads, 128] bf16, element strides (kv_stride_token, kv_stride_head)
 *   out [q_len,  num_qo_heads, 128] bf16, element strides (out_stride_token, out_stride_head)
 * Strides must be multiples of 8 elements and pointers 16-byte aligned (TMA). With causal != 0,
 * query i attends keys j <= kv_len - q_len + i (bottom-right alignment; q_len <= kv_len): the
 * square causal prefill when q_len == kv_len. Query head h reads KV head h / (nqo / nkv).
 * Replaces src/solort/model/cuda_graph_executor.py:124-130 (repeat_interleave + causal SDPA) and
 * src/solort/backends/transformers_flashinfer.py:114-129 (FlashInfer single_prefill, causal).
 */
typedef struct SolortPrefillArgs {
  const void* q;
  int64_t q_stride_token, q_stride_head;
  const void* k;
  const void* v;
  int64_t kv_stride_token, kv_stride_head;
  void* out;
  int64_t out_stride_token, out_stride_head;
  int32_t q_len, kv_len, num_qo_heads, num_kv_heads, head_dim;
  int32_t causal;
  float scale;
} SolortPrefillArgs;

SOLORT_API int solort_attn_prefill(const SolortPrefillArgs* args, void* stream);

/*
 * Attention prologue of one layer (decode, verify or prefill): per-head QK-RMSNorm and rotate-half
 * RoPE of the fused QKV projection, the normalised queries written to q_out, and this step's K / V
 * rows appended to the cache. Replaces src/solort/model/cuda_graph_executor.py:176-179 (decode),
 * :120-123 (prefill) and :257-260 (verify): _rmsnorm (:25-28), _rope (:100-102) with the bf16
 * _cos_sin tables (:95-98), and the index_copy_ / slice stores into kc/vc; with a block table, the
 * slot-mapped store of src/solort/cache/kv_cache.py:136-149,191-235.
 *   qkv      [num_tokens, (nqo + 2*nkv) * 128] bf16: query heads, then key heads, then value heads
 *   q/k_norm_weight [128] bf16; eps as the model's rms_norm_eps
 *   cos, sin [rope_rows, 128] bf16: the model's tables by position (row p = _cos_sin(p))
 *   pos      int64 [1] on the device: token i sits at position pos[0] + i
 *   q_out    token i, head h at q_out + i*q_out_stride_token + h*q_out_stride_head (bf16)
 *   k/v_cache static: row (position p, kv head h) at + p*kv_stride_token + h*kv_stride_head,
 *            kv_capacity rows; paged (block_table != NULL): page bt[p / page_size], row
 *            p % page_size at + page*kv_stride_page + row*kv_stride_token + h*kv_stride_head,
 *            kv_capacity = num_pages * page_size. Positions past kv_capacity are not stored.
 * Rounding follows the reference step by step except the fp32 sum of squares, a warp tree.
 * Pointers 8-byte aligned, strides multiples of 4 elements.
 */
typedef struct SolortPrologueArgs {
  const void* qkv;
  int64_t qkv_stride_token;
  int32_t num_tokens, num_qo_heads, num_kv_heads, head_dim;
  const void* q_norm_weight;
  const void* k_norm_weight;
  float eps;
  const void* cos;
  const void* sin;
  int64_t rope_stride;
  int32_t rope_rows;
  const int64_t* pos;
  void* q_out;
  int64_t q_out_stride_token, q_out_stride_head;
  void* k_cache;
  void* v_cache;
  int64_t kv_stride_token, kv_stride_head, kv_stride_page;
  int32_t kv_capacity;
  const int32_t* block_table;
  int32_t page_size;
} SolortPrologueArgs;

SOLORT_API int solort_attn_qk_norm_rope_append(const SolortPrologueArgs* args, void* stream);

/*
 * Slot-mapped store of num_tokens tokens' K and V rows into a paged arena: token i goes to
 * physical slot slots[i] = page * page_size + row. Replaces the per-token Python loop of
 * PagedKVCache.store_layer_tokens (src/solort/cache/kv_cache.py:191-235), which the HF bridge
 * calls to mirror each layer's K / V (src/solort/backends/transformers_flashinfer.py:93,205-220).
 *   key, value  token i, kv head h at key + i*src_stride_token + h*src_stride_head (bf16, the 128
 *               dims contiguous); for the HF layout [1, nkv, kv, 128] pass the last num_tokens
 *               tokens' base with src_stride_token = 128 and src_stride_head = kv * 128
 *   slots       int64 [num_tokens] on the device
 *   k_pages, v_pages  row (page p, row r, head h) at + p*dst_stride_page + r*dst_stride_token +
 *               h*dst_stride_head; for SoloRT's arena [pages, 2, P, nkv, 128]: v_pages = k_pages +
 *               P*nkv*128, dst_stride_page = 2*P*nkv*128
 * Copies are bit-exact. A slot outside [0, num_pages * page_size) is skipped and sets bit 4 of the
 * device status. Pointers 16-byte aligned, strides multiples of 8 elements.
 */
typedef struct SolortKVStoreArgs {
  const void* key;
  const void* value;
  int64_t src_stride_token, src_stride_head;
  int32_t num_tokens, num_kv_heads, head_dim;
  const int64_t* slots;
  void* k_pages;
  void* v_pages;
  int64_t dst_stride_page, dst_stride_token, dst_stride_head;
  int32_t page_size, num_pages;
} SolortKVStoreArgs;

SOLORT_API int solort_attn_kv_store(const SolortKVStoreArgs* args, void* stream);

/*
 * Layer glue of the runner's step (decode, verify or prefill) around the attention.
 * solort_attn_add_rmsnorm: per row, x_out = x + delta (bf16, when delta != NULL; x_out may be x),
 * then h_out = RMSNorm(x_out) * weight: fp32 x * rsqrt(mean(x^2) + eps), times the weight, cast to
 * bf16 -- the reference's _rmsnorm (src/solort/model/cuda_graph_executor.py:25-28) after the
 * layer loop's residual add; the fp32 sum of squares is a tree. hidden a multiple of 8 and at most
 * 16384; pointers 16-byte aligned, strides (elements) multiples of 8.
 * solort_attn_silu_mul: out[r, i] = bf16(bf16(silu(g)) * u) with g = gate_up[r, i] and
 * u = gate_up[r, inter + i] -- the MLP's F.silu(gate) * up on the fused gate/up projection.
 */
typedef struct SolortAddRmsNormArgs {
  const void* x;
  int64_t x_stride;
  const void* delta; /* optional */
  int64_t delta_stride;
  const void* weight;
  void* x_out;
  int64_t x_out_stride;
  void* h_out;
  int64_t h_out_stride;
  int32_t rows, hidden;
  float eps;
} SolortAddRmsNormArgs;

SOLORT_API int solort_attn_add_rmsnorm(const SolortAddRmsNormArgs* args, void* stream);

typedef struct SolortSiluMulArgs {
  const void* gate_up;
  int64_t gate_up_stride;
  void* out;
  int64_t out_stride;
  int32_t rows, inter;
} SolortSiluMulArgs;

SOLORT_API int solort_attn_silu_mul(const SolortSiluMulArgs* args, void* stream);

/*
 * Weight-streaming projection for the decode step (t <= 8 token rows), replacing the runner's
 * torch matmuls against a bf16 Linear weight W [n, k] (row stride w_stride):
 *   y[r, j] = bf16( sum_i act[r, i] * W[j, i] )   (fp32 accumulation)
 * mode 0: act = a [t, k];
 * mode 1: act = bf16(bf16(silu(g)) * u) with g = a[r, 0:k], u = a[r, k:2k] (the MLP's
 *         F.silu(gate) * up fused into the down projection);
 * mode 2: act = RMSNorm(x) * norm_weight with x = a (the residual stream) or, when delta is given,
 *         x = bf16(a + delta), which is also written to x_out (the residual add and the norm after
 *         it, bit-identical to solort_attn_add_rmsnorm); x_out must not overlap a or delta.
 * W is read before the kernel waits for the previous kernel on the stream (PDL), so it must not be
 * written by that kernel. k a multiple of 8, t * k * 2 bytes staged per CTA at most 160 KB;
 * pointers 16-byte aligned, strides multiples of 8 elements.
 * Reference: src/solort/model/cuda_graph_executor.py _rmsnorm :25-28 and the layer loop's
 * projections (:168-190).
 */
typedef struct SolortGemvArgs {
  const void* a;
  int64_t a_stride;
  const void* w;
  int64_t w_stride;
  void* y;
  int64_t y_stride;
  int32_t t, n, k, mode;
  const void* delta;        /* mode 2, optional */
  int64_t delta_stride;
  const void* norm_weight;  /* mode 2: [k] */
  void* x_out;              /* mode 2 with delta */
  int64_t x_out_stride;
  float eps;
} SolortGemvArgs;

SOLORT_API int solort_attn_gemv(const SolortGemvArgs* args, void* stream);

/* Reads and clears the device status word of the current device (bit 0: an in-kernel wait hit
 * its time limit and the kernel returned without writing its output; bit 1: a tensor-memory
 * allocation wait hit its limit; bit 2: a kernel found its shared memory misaligned and returned
 * without writing; bit 3: an exchange merge waited a second for a peer's partial and left the
 * row unwritten; bit 4: solort_attn_kv_store met a slot outside the arena and skipped it). */
SOLORT_API int solort_attn_device_status(unsigned* flags);

SOLORT_API const char* solort_attn_status_string(int code);
SOLORT_API int solort_attn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SOLORT_ATTN_H_ */
