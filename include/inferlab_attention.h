/*
 * inferlab_attention.h - C ABI of the B200 (sm_100a) attention library.
 *
 * Two groups of entry points:
 *
 *  1. The reference worker's attention entry, same signature and semantics:
 *     inferlab_attention_forward() replaces the CPU implementation declared at
 *     worker/cpp/inferlab_runtime.h:216-231 (implemented at
 *     worker/cpp/inferlab_runtime.cpp:2561-2619 on top of
 *     kernels/attention_cpu.cpp:419-502). Host buffers in, host buffer out;
 *     the copies to and from HBM happen inside the call.
 *
 *  2. A device-resident paged KV pool and the kernels that read it through
 *     block tables. They replace PagedKvPool's page storage, append and
 *     materialize (worker/cpp/inferlab_runtime.cpp:649-1026) and the per-step
 *     gather + attention_forward call of the paged decode branch
 *     (worker/cpp/inferlab_runtime.cpp:2373-2393). Block-table semantics are
 *     the reference's: logical block = position / block_tokens,
 *     slot = position % block_tokens, physical block = table[logical block].
 *     All pointers marked "device" are HBM pointers on the pool's device; all
 *     calls are asynchronous on the given stream (NULL = the legacy default
 *     stream) and take a cudaStream_t passed as void*.
 *
 * Error convention (both groups), as worker/cpp/inferlab_runtime.cpp:2013-2030:
 * functions return 0 on success and -1 on failure, writing a NUL-terminated
 * message truncated to error_capacity into `error` (which is cleared on entry).
 * Host-side argument errors are reported by the call itself. Errors found by a
 * kernel (a non-finite row, a block id outside the pool, an invalid
 * normaliser) are recorded in the pool's device error word and reported by the
 * next inferlab_cuda_pool_synchronize() on that pool.
 */
#ifndef INFERLAB_ATTENTION_H
#define INFERLAB_ATTENTION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* worker/cpp/inferlab_runtime.h:67-72 (field meaning from
 * kernels/attention_cpu.h:8-24): algorithm 0 Materialized / 1 OnlineTiled,
 * precision 0 Fp32 / 1 Fp16 / 2 Bf16 storage rounding, tile_tokens 1..4096,
 * causal 0/1. */
typedef struct InferlabAttentionConfig {
    uint32_t algorithm;
    uint32_t precision;
    uint32_t tile_tokens;
    uint32_t causal;
} InferlabAttentionConfig;

/* worker/cpp/inferlab_runtime.h:74-83; analytic counters computed exactly as
 * kernels/attention_cpu.cpp:140-213 (they model the reference CPU algorithm;
 * the CUDA kernels' own traffic is measured, not modelled). */
typedef struct InferlabAttentionStats {
    uint64_t score_elements;
    uint64_t masked_score_elements;
    uint64_t score_buffer_bytes;
    uint64_t working_set_bytes;
    uint64_t modeled_external_read_bytes;
    uint64_t modeled_external_write_bytes;
    uint64_t modeled_external_total_bytes;
    uint64_t key_tiles;
} InferlabAttentionStats;

/*
 * Replaces inferlab_attention_forward, worker/cpp/inferlab_runtime.h:216-231.
 * queries [query_tokens][heads][head_dimension], keys/values
 * [key_value_tokens][heads][head_dimension], output likewise for queries; all
 * fp32 host memory. Validation order and messages follow
 * worker/cpp/inferlab_runtime.cpp:2578-2593 and kernels/attention_cpu.cpp:432-447.
 * Runs on the calling thread's current CUDA device. Both algorithms run the
 * same fused online-softmax kernel in fp32 (storage rounding applied on load);
 * the output matches either CPU algorithm within 1e-5 relative / 1e-6 absolute.
 * Exception: causal calls in the Fp16 / Bf16 storage modes with head_dimension
 * 128 and at least 1024 query rows (query_tokens x heads; the full-prompt call
 * of Model::forward_all, worker/cpp/inferlab_runtime.cpp:1327-1339) run on the
 * tensor cores with fp16 probabilities: within 2e-3 relative plus 1e-3 of the
 * row's largest output. Inputs whose rounded values leave fp16's range (bf16
 * V above 65504, fp16 overflow) fall back to the fp32 kernel. Stats are
 * exact either way. head_dimension is limited to 4096 on the device.
 */
int inferlab_attention_forward(const float* queries, const float* keys, const float* values,
                               size_t query_tokens, size_t key_value_tokens, size_t heads,
                               size_t head_dimension, size_t query_start_position,
                               const InferlabAttentionConfig* config, float* output,
                               size_t output_capacity, InferlabAttentionStats* stats,
                               char* error, size_t error_capacity);

/* ------------------------------------------------------------------------ */
/* Device-resident paged KV pool                                             */
/* ------------------------------------------------------------------------ */

/* Element type of a pool (same numbering as the attention precision). */
#define INFERLAB_KV_FP32 0u
#define INFERLAB_KV_F16 1u
#define INFERLAB_KV_BF16 2u

typedef struct InferlabCudaKvPool InferlabCudaKvPool;

/* Geometry and device addresses of a pool. Each arena is
 * [num_blocks][kv_heads][block_tokens][head_dim] elements of `dtype`: one
 * block of one kv-head is a contiguous block_tokens x head_dim tile. */
typedef struct InferlabCudaPoolInfo {
    int32_t device;
    uint32_t dtype;
    uint32_t block_tokens;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t element_bytes;
    uint64_t num_blocks;
    uint64_t block_bytes;  /* bytes of one block in one arena, all kv-heads */
    uint64_t arena_bytes;  /* bytes of one arena */
    void* key_arena;       /* device */
    void* value_arena;     /* device */
} InferlabCudaPoolInfo;

/*
 * Allocates a pool of num_blocks blocks in HBM on `device` (the device pool
 * behind PagedKvPool's page storage, worker/cpp/inferlab_runtime.cpp:657-678,
 * configured like inferlab_model_configure_paged_cache, :2157-2189; the
 * reference's 65,536-page cap is lifted because HBM holds ~180 GB). The arenas
 * are zero-filled. Block ids are int32, so num_blocks < 2^31.
 */
int inferlab_cuda_pool_create(int32_t device, uint32_t dtype, uint64_t num_blocks,
                              uint32_t block_tokens, uint32_t kv_heads, uint32_t head_dim,
                              InferlabCudaKvPool** pool, char* error, size_t error_capacity);

/* Frees the arenas (after synchronising the device). NULL is a no-op. */
void inferlab_cuda_pool_destroy(InferlabCudaKvPool* pool);

int inferlab_cuda_pool_info(const InferlabCudaKvPool* pool, InferlabCudaPoolInfo* info,
                            char* error, size_t error_capacity);

/*
 * Waits for `stream` for at most timeout_ms milliseconds (0 = 10 s), then
 * reads and clears the pool's device error word. Returns -1 with the first
 * recorded error ("paged KV block table contains an invalid page",
 * "attention input must be finite", "online attention normalizer is
 * invalid", "paged KV context length is invalid", ...) or with
 * "CUDA stream wait timed out" when the stream is still busy.
 */
int inferlab_cuda_pool_synchronize(InferlabCudaKvPool* pool, void* stream, uint32_t timeout_ms,
                                   char* error, size_t error_capacity);

/*
 * Writes `rows` token rows into the pool (the data movement of
 * PagedKvPool::append, worker/cpp/inferlab_runtime.cpp:713-767, without its
 * host-side allocation policy). Row r is key_rows[r] / value_rows[r], each
 * [kv_heads][head_dim] of `row_dtype` (INFERLAB_KV_FP32, rounded to the pool
 * type like round_attention_value, kernels/attention_cpu.cpp:405-417; or the
 * pool's own type, copied bit for bit), and goes to position positions[r] of
 * sequence row_sequences[r]: block block_tables[seq * max_blocks_per_seq +
 * pos / block_tokens], slot pos % block_tokens. Non-finite values are
 * rejected ("attention input must be finite"); the row is not written.
 * All arrays are device memory.
 */
int inferlab_cuda_kv_append(InferlabCudaKvPool* pool, const void* key_rows, const void* value_rows,
                            uint32_t row_dtype, const int32_t* row_sequences,
                            const int32_t* positions, uint64_t rows, const int32_t* block_tables,
                            uint32_t max_blocks_per_seq, void* stream, char* error,
                            size_t error_capacity);

/*
 * The Q/K/V projection beside attention, with the K/V rows appended in the
 * same launch: the three fp32 `linear` calls of the reference's forward pass
 * (worker/cpp/inferlab_runtime.cpp:1318-1325, linear at :1266-1285) plus the
 * PagedKvPool::append of their K/V rows (:713-767), on the tensor cores.
 * hidden [tokens][model_dim] and weights [(q_heads + 2 kv_heads) head_dim]
 * [model_dim] (the stacked W_q, W_k, W_v, one output feature per row) are in
 * the pool's type (F16 or BF16 pools); products accumulate in fp32 and are
 * rounded to the pool type. Q goes to q_out [tokens][q_heads][head_dim] (pool
 * type); token t's K and V rows go to position positions[t] of sequence
 * row_sequences[t] (< num_seqs) through block_tables [num_seqs]
 * [max_blocks_per_seq]. head_dim must be a multiple of 32, model_dim of 8;
 * hidden, weights and q_out 16-byte aligned. Device memory, asynchronous on
 * `stream`; a bad position or block id ("paged KV append position is outside
 * the block table", "paged KV block table contains an invalid page") skips
 * that token's K/V rows, a non-finite K/V value is reported ("attention input
 * must be finite") - both through the pool's error word.
 */
int inferlab_cuda_qkv_project_append(InferlabCudaKvPool* pool, const void* hidden,
                                     const void* weights, uint32_t tokens, uint32_t model_dim,
                                     uint32_t q_heads, const int32_t* row_sequences,
                                     const int32_t* positions, const int32_t* block_tables,
                                     uint32_t num_seqs, uint32_t max_blocks_per_seq, void* q_out,
                                     void* stream, char* error, size_t error_capacity);

/*
 * The output projection after attention, with the residual add: the
 * reference's `linear(attention_context, ..., attention_output_weight, ...)`
 * and `hidden += attention_output` (worker/cpp/inferlab_runtime.cpp:
 * 1340-1350), on the tensor cores. attention [tokens][in_dim] (fp32, as the
 * attention entries return it, rounded here to the pool type; or already in
 * the pool type), weights [out_dim][in_dim] in the pool's type (F16 / BF16
 * pools; the pool supplies the device and the error word), residual
 * [tokens][out_dim] fp32 or NULL, out [tokens][out_dim] fp32 = residual +
 * attention x weights^T with fp32 accumulation. in_dim a multiple of 8,
 * out_dim of 32; buffers 16-byte aligned; device memory, asynchronous.
 */
int inferlab_cuda_output_project(InferlabCudaKvPool* pool, const void* attention,
                                 uint32_t attention_dtype, const void* weights,
                                 const float* residual, uint32_t tokens, uint32_t in_dim,
                                 uint32_t out_dim, float* out, void* stream, char* error,
                                 size_t error_capacity);

/*
 * Copies the first `tokens` positions of one sequence into contiguous
 * [tokens][kv_heads][head_dim] arrays of the pool's type, bit for bit: the
 * device form of PagedKvPool::materialize (worker/cpp/inferlab_runtime.cpp:
 * 769-803). block_table holds ceil(tokens / block_tokens) device int32 ids.
 */
int inferlab_cuda_kv_gather(InferlabCudaKvPool* pool, const int32_t* block_table, uint64_t tokens,
                            void* keys_out, void* values_out, void* stream, char* error,
                            size_t error_capacity);

/*
 * Bytes of device workspace inferlab_cuda_paged_decode needs for this batch
 * shape. max_context_len bounds every context_lens[i].
 */
size_t inferlab_cuda_paged_decode_workspace_size(const InferlabCudaKvPool* pool, uint32_t num_seqs,
                                                 uint32_t q_heads, uint32_t max_context_len);

/*
 * Fixes the decode split length of this pool's later decode calls at
 * blocks_per_split 16-token blocks (1..1024; 0 restores the planner's own
 * choice, the default). The planner still caps a split at 256 blocks and a
 * context at 64 splits. A tuning and test setting with no counterpart in the
 * reference (its decode is one host call per sequence); workspace sizes
 * follow it, so query inferlab_cuda_paged_decode_workspace_size after
 * changing it. Not synchronised with decode calls on other host threads.
 */
int inferlab_cuda_pool_set_decode_split(InferlabCudaKvPool* pool, uint32_t blocks_per_split,
                                        char* error, size_t error_capacity);

/*
 * Zeroes the counters at the front of a decode workspace. Needed once per
 * workspace before its first use; the decode kernel leaves them at zero.
 */
int inferlab_cuda_paged_decode_workspace_init(void* workspace, size_t workspace_bytes,
                                              void* stream, char* error, size_t error_capacity);

/*
 * One decode step for a batch: sequence i has one query token at position
 * context_lens[i] - 1 attending to positions [0, context_lens[i]) of its
 * block table row (the call shape of worker/cpp/inferlab_runtime.cpp:
 * 1458-1470, attention_forward(q, K, V, 1, T, H, d, T - 1)).
 * queries: device fp32 [num_seqs][q_heads][head_dim], rounded to the pool's
 * type on load (the reference's Fp16/Bf16 storage modes round queries too).
 * q-head h reads kv-head h / (q_heads / kv_heads) (grouped-query attention;
 * q_heads must be a multiple of kv_heads). block_tables: device int32
 * [num_seqs][max_blocks_per_seq]. context_lens: device int32 [num_seqs],
 * each in [1, max_context_len] and <= max_blocks_per_seq * block_tokens.
 * out: device fp32 [num_seqs][q_heads][head_dim]. Long contexts are split
 * across CTAs and merged by log-sum-exp inside the same launch; workspace
 * (inferlab_cuda_paged_decode_workspace_size bytes, initialised once with
 * inferlab_cuda_paged_decode_workspace_init) holds the split partials.
 */
int inferlab_cuda_paged_decode(InferlabCudaKvPool* pool, const float* queries,
                               const int32_t* block_tables, uint32_t max_blocks_per_seq,
                               const int32_t* context_lens, uint32_t num_seqs, uint32_t q_heads,
                               uint32_t max_context_len, float* out, void* workspace,
                               size_t workspace_bytes, void* stream, char* error,
                               size_t error_capacity);

/*
 * inferlab_cuda_paged_decode without a caller workspace, for callers that
 * cannot allocate device memory (for example a process whose GPU memory is
 * reserved up front by another framework's allocator, or a serving loop that
 * may not call cudaMalloc once running). No counterpart in the reference,
 * whose decode runs on the host. The split-KV scratch is a 16 MiB array built
 * into the library (held by every GPU that loads it until the process exits);
 * batches whose split partials need more than that are rejected with an error
 * naming the size, while batches with one split per sequence need no scratch
 * at any size. The call allocates nothing. Calls share the array: two calls
 * whose work overlaps on the GPU race, so serialise them. The first call on a
 * device that needs scratch looks up the array's device address and caches
 * it; make it before any stream capture, and do not call this entry after a
 * device reset (the cached address goes stale). Arguments as
 * inferlab_cuda_paged_decode.
 */
int inferlab_cuda_paged_decode_noalloc(InferlabCudaKvPool* pool, const float* queries,
                                       const int32_t* block_tables, uint32_t max_blocks_per_seq,
                                       const int32_t* context_lens, uint32_t num_seqs,
                                       uint32_t q_heads, uint32_t max_context_len, float* out,
                                       void* stream, char* error, size_t error_capacity);

/*
 * One continuous-batching decode step with HOST buffers, synchronous: the
 * per-sequence append + materialize + attention_forward loop of the
 * reference's paged decode (worker/cpp/inferlab_runtime.cpp:2373-2393 driven
 * by worker/src/scheduler.rs:268-270) for a whole batch in one call.
 * queries [num_seqs][q_heads][head_dim], new_keys / new_values
 * [num_seqs][kv_heads][head_dim] (both NULL to skip the append), block_tables
 * [num_seqs][max_blocks_per_seq], context_lens [num_seqs] (the new token sits
 * at position context_lens[i] - 1 and attends to [0, context_lens[i])), out
 * [num_seqs][q_heads][head_dim]; all host memory, fp32 / int32. When every
 * array is page-locked (cudaHostAlloc / cudaHostRegister) a prologue kernel
 * reads them over the bus, appending the new rows and staging the decode's
 * inputs, and the decode writes straight into `out`: two launches and a
 * 4-byte copy. Otherwise the inputs cross to HBM by copies (through the
 * pool's pinned staging for pageable arrays), then kv_append, one decode
 * launch, one copy back. Waits at most timeout_ms (0 = 10 s). Context lengths
 * are checked on the host first; block ids where the append and decode kernels
 * read them, failing the call with the same message (the reference's
 * materialize checks, :776-789).
 */
int inferlab_cuda_decode_step_host(InferlabCudaKvPool* pool, const float* queries,
                                   const float* new_keys, const float* new_values,
                                   const int32_t* block_tables, uint32_t max_blocks_per_seq,
                                   const int32_t* context_lens, uint32_t num_seqs,
                                   uint32_t q_heads, float* out, void* stream,
                                   uint32_t timeout_ms, char* error, size_t error_capacity);

/*
 * inferlab_cuda_decode_step_host with the step's copy-on-write block copies
 * fused in: block_copies [num_seqs][2] holds, per sequence, the (from, to)
 * block pair inferlab_cuda_pages_prepare_append returned for this append
 * (PagedKvPool::append, worker/cpp/inferlab_runtime.cpp:738-754), or
 * (-1, -1). Each copy (both arenas, the whole block) completes before that
 * sequence's new row is written; with page-locked arrays the copies run in
 * the step's prologue kernel. Needs new_keys / new_values.
 */
int inferlab_cuda_decode_step_host_cow(InferlabCudaKvPool* pool, const float* queries,
                                       const float* new_keys, const float* new_values,
                                       const int32_t* block_copies, const int32_t* block_tables,
                                       uint32_t max_blocks_per_seq, const int32_t* context_lens,
                                       uint32_t num_seqs, uint32_t q_heads, float* out,
                                       void* stream, uint32_t timeout_ms, char* error,
                                       size_t error_capacity);

/*
 * Decode partials for a context that is split across devices: like
 * inferlab_cuda_paged_decode, but instead of the normalised output it writes,
 * per (sequence, q-head) row r = seq * q_heads + h,
 *   part_m[r] = max score (natural-log units, scores already scaled by
 *               1/sqrt(head_dim)),
 *   part_l[r] = sum exp(score - part_m[r]),
 *   part_o[r][d] = sum exp(score - part_m[r]) * v[d]   (unnormalised),
 * over every position the block table row covers (all of them are visible to
 * the query: it sits after the whole local range). Rows with no keys get
 * m = -inf, l = 0, o = 0. The parts are merged with inferlab_cuda_lse_combine.
 */
int inferlab_cuda_paged_decode_partials(InferlabCudaKvPool* pool, const float* queries,
                                        const int32_t* block_tables, uint32_t max_blocks_per_seq,
                                        const int32_t* context_lens, uint32_t num_seqs,
                                        uint32_t q_heads, uint32_t max_context_len, float* part_m,
                                        float* part_l, float* part_o, void* workspace,
                                        size_t workspace_bytes, void* stream, char* error,
                                        size_t error_capacity);

/*
 * Log-sum-exp merge of `parts` partial results in part order (deterministic):
 * part_m, part_l [parts][rows], part_o [parts][rows][head_dim], all device fp32;
 * out [rows][head_dim] = sum_i o_i e^(m_i - M) / sum_i l_i e^(m_i - M),
 * M = max over parts with l_i > 0.
 */
int inferlab_cuda_lse_combine(const float* part_m, const float* part_l, const float* part_o,
                              uint32_t parts, uint64_t rows, uint32_t head_dim, float* out,
                              void* stream, char* error, size_t error_capacity);

/*
 * The same merge over `parts` packed partials, part i at
 * packed + i * rows * (head_dim + 2) laid out as [m: rows][l: rows]
 * [o: rows][head_dim] - one block per rank as a single all-gather of
 * [m | l | o] delivers them (inferlab_cuda_paged_decode_partials can write the
 * three pieces of the local block directly). No reference counterpart.
 */
int inferlab_cuda_lse_combine_packed(const float* packed, uint32_t parts, uint64_t rows,
                                     uint32_t head_dim, float* out, void* stream, char* error,
                                     size_t error_capacity);

/*
 * Causal prefill / chunked prefill over the paged pool. Segment s has
 * query_counts[s] query tokens at positions [query_starts[s],
 * query_starts[s] + query_counts[s]) of its sequence, whose keys and values
 * for positions [0, query_starts[s] + query_counts[s]) are already in the
 * pool under block table row s; query i attends to positions
 * [0, query_starts[s] + i] (legal_sources, kernels/attention_cpu.cpp:113-123).
 * queries: device [total_queries][q_heads][head_dim] of query_dtype
 * (INFERLAB_KV_FP32 is rounded to the pool type; otherwise it must equal the
 * pool type); segment s uses rows [query_offsets[s], query_offsets[s] +
 * query_counts[s]), and the segments tile [0, total_queries) in order.
 * query_starts, query_counts, query_offsets: device int32 [num_segments].
 * out: device fp32 [total_queries][q_heads][head_dim].
 * f16/bf16 pools with head_dim 128 and block_tokens 16 run on the tcgen05
 * tensor cores (fp32 accumulation in TMEM); other pools run a fp32 CUDA-core
 * kernel. max_query_count bounds every query_counts[s].
 */
int inferlab_cuda_paged_prefill(InferlabCudaKvPool* pool, const void* queries, uint32_t query_dtype,
                                const int32_t* block_tables, uint32_t max_blocks_per_seq,
                                const int32_t* query_starts, const int32_t* query_counts,
                                const int32_t* query_offsets, uint32_t num_segments,
                                uint32_t q_heads, uint32_t max_query_count,
                                uint64_t total_queries, float* out, void* stream, char* error,
                                size_t error_capacity);

/* ---- Block ownership (host metadata over the device pool) -------------------
 *
 * The ownership model of the reference's PagedKvPool
 * (worker/cpp/inferlab_runtime.cpp:649-1032) without its page storage, which
 * lives in the device pool: a free list, reference counts, published prefixes
 * with longest-prefix lookup and least-recently-used eviction, copy on write
 * for a shared tail block, and InferlabPagedCacheStats. Block ids are the
 * device pool's. All calls are host-only except inferlab_cuda_pages_copy.
 */
#ifndef INFERLAB_PAGED_CACHE_STATS_DEFINED
#define INFERLAB_PAGED_CACHE_STATS_DEFINED
/* Same layout and meaning as worker/cpp/inferlab_runtime.h:7-31. */
typedef struct InferlabPagedCacheStats {
    uint64_t page_tokens;
    uint64_t page_count;
    uint64_t prefix_capacity;
    uint64_t page_bytes;
    uint64_t capacity_bytes;
    uint64_t allocated_pages;
    uint64_t free_pages;
    uint64_t used_token_slots;
    uint64_t allocated_token_slots;
    uint64_t internal_fragmentation_bytes;
    uint64_t live_references;
    uint64_t shared_pages;
    uint64_t maximum_refcount;
    uint64_t logical_referenced_bytes;
    uint64_t physical_used_bytes;
    uint64_t bytes_saved_by_sharing;
    uint64_t prefix_entries;
    uint64_t prefix_hits;
    uint64_t prefix_misses;
    uint64_t prefix_tokens_reused;
    uint64_t copy_on_write_copies;
    uint64_t evictions;
    uint64_t allocation_failures;
} InferlabPagedCacheStats;
#endif

typedef struct InferlabCudaPageManager InferlabCudaPageManager;

/*
 * A manager of page_count blocks of block_tokens token rows; row_bytes is one
 * token row of K and V over all kv-heads (kv_heads * head_dim * 2 * element
 * bytes), so page_bytes = block_tokens * row_bytes. Replaces PagedKvPool's
 * constructor (:656-677; "paged KV cache dimensions must be positive").
 */
int inferlab_cuda_pages_create(uint64_t page_count, uint32_t block_tokens, uint64_t row_bytes,
                               uint64_t prefix_capacity, InferlabCudaPageManager** manager,
                               char* error, size_t error_capacity);
void inferlab_cuda_pages_destroy(InferlabCudaPageManager* manager);

/*
 * Reserves the slot of token `cached_tokens` of a sequence whose block table
 * is table[0 .. *table_length) (ceil(cached_tokens / block_tokens) entries,
 * room for table_capacity): a new block when the slot starts one, else the
 * tail block, copied first when it is shared - *copy_from / *copy_to name the
 * blocks the caller copies on the device (inferlab_cuda_pages_copy) before it
 * writes the row; both are -1 when no copy is needed. The allocation policy of
 * PagedKvPool::append (:710-767), whose row write is inferlab_cuda_kv_append.
 */
int inferlab_cuda_pages_prepare_append(InferlabCudaPageManager* manager, int32_t* table,
                                       uint32_t table_capacity, uint32_t* table_length,
                                       uint64_t cached_tokens, int32_t* copy_from,
                                       int32_t* copy_to, char* error, size_t error_capacity);

/* Drops one reference on each block of the table (PagedKvPool::release_table, :848-855). */
int inferlab_cuda_pages_release(InferlabCudaPageManager* manager, const int32_t* table,
                                uint32_t length, char* error, size_t error_capacity);

/* PagedKvPool::publish_prefix (:805-846): the first ceil(token_count / block_tokens) blocks. */
int inferlab_cuda_pages_publish_prefix(InferlabCudaPageManager* manager, const uint32_t* tokens,
                                       uint64_t token_count, const int32_t* table, uint32_t length,
                                       uint64_t cached_tokens, char* error, size_t error_capacity);

/*
 * PagedKvPool::acquire_longest_prefix (:679-708): the longest published prefix
 * of tokens, its blocks retained for the caller and written to table;
 * *prefix_tokens = 0 and *table_length = 0 on a miss.
 */
int inferlab_cuda_pages_acquire_prefix(InferlabCudaPageManager* manager, const uint32_t* tokens,
                                       uint64_t token_count, int32_t* table,
                                       uint32_t table_capacity, uint32_t* table_length,
                                       uint64_t* prefix_tokens, char* error, size_t error_capacity);

/* PagedKvPool::shared_pages (:857-867): blocks of the table with more than one reference. */
int inferlab_cuda_pages_shared(InferlabCudaPageManager* manager, const int32_t* table,
                               uint32_t length, uint64_t* shared, char* error,
                               size_t error_capacity);

/* PagedKvPool::stats (:877-911) with the device pool's block and row sizes. */
int inferlab_cuda_pages_stats(InferlabCudaPageManager* manager, InferlabPagedCacheStats* stats,
                              char* error, size_t error_capacity);

/*
 * Copies whole blocks from[i] -> to[i] (K and V arenas, all kv-heads) on
 * `stream`: the data movement of the copy on write (:741-750).
 */
int inferlab_cuda_pages_copy(InferlabCudaKvPool* pool, const int32_t* from, const int32_t* to,
                             uint32_t count, void* stream, char* error, size_t error_capacity);

/*
 * Peer exchange of split-KV partials (one process per GPU, GPUs of one box
 * connected by NVLink): the all-gather of the packed [m | l | o] blocks and
 * inferlab_cuda_lse_combine_packed in ONE kernel. Each rank allocates its
 * receive buffer (inferlab_cuda_peer_buffer_alloc, which also returns the
 * buffer's CUDA IPC handle), the ranks swap handles over their own process
 * group, and inferlab_cuda_peer_exchange_create opens the peers' buffers.
 * Per call the kernel stores this rank's block into slot `rank` of every
 * peer's buffer (peer stores over NVLink, no multicast; every element as one
 * 8-byte word with the step number in its high half, so no separate flag or
 * fence is needed), waits (bounded, ~2 s) until every rank's words of this
 * step have arrived in its own buffer, and merges the blocks in rank order,
 * bit for bit as inferlab_cuda_lse_combine_packed would. The words alternate
 * between two slots by step parity, so a rank one step ahead never overwrites
 * a block a peer is still reading. A wait that gives up records "device wait
 * timed out", read by inferlab_cuda_peer_exchange_synchronize.
 * Every rank must call the same sequence of exchanges, and each rank's
 * exchanges must run one after another on the GPU (one stream, or streams
 * ordered by events): the parity argument above holds only when a rank's
 * exchange s + 2 starts after its exchange s + 1 has finished. No reference
 * counterpart (the reference has no split-sequence decode).
 */
typedef struct InferlabCudaPeerExchange InferlabCudaPeerExchange;

#define INFERLAB_CUDA_IPC_HANDLE_BYTES 64u
#define INFERLAB_CUDA_PEER_MAX_RANKS 8u

/* Bytes of one rank's receive buffer for `world` ranks and `rows` rows. */
uint64_t inferlab_cuda_peer_buffer_bytes(uint32_t world, uint64_t rows, uint32_t head_dim);

/* Allocates and zeroes a receive buffer on `device`; writes its IPC handle
 * (INFERLAB_CUDA_IPC_HANDLE_BYTES bytes) to handle. */
int inferlab_cuda_peer_buffer_alloc(int device, uint64_t bytes, void** buffer, void* handle,
                                    char* error, size_t error_capacity);
int inferlab_cuda_peer_buffer_free(int device, void* buffer, char* error, size_t error_capacity);

/* handles: world x INFERLAB_CUDA_IPC_HANDLE_BYTES, rank r's at r (this rank's
 * own entry is ignored); local_buffer: this rank's buffer. Each exchange
 * counts its steps from 1 and the buffers keep the last step-tagged words, so
 * every exchange needs buffers fresh from inferlab_cuda_peer_buffer_alloc
 * (zeroed): an exchange created again on buffers an earlier one used could
 * take that one's words for its own. */
int inferlab_cuda_peer_exchange_create(int device, uint32_t world, uint32_t rank, uint64_t rows,
                                       uint32_t head_dim, void* local_buffer, const void* handles,
                                       InferlabCudaPeerExchange** out, char* error,
                                       size_t error_capacity);

/* packed: this rank's [m | l | o] block (rows x (head_dim + 2) fp32, device);
 * out: [rows][head_dim] fp32 (device). Asynchronous on `stream`. */
int inferlab_cuda_peer_exchange_combine(InferlabCudaPeerExchange* exchange, const float* packed,
                                        float* out, void* stream, char* error,
                                        size_t error_capacity);

/* Waits for `stream` (bounded) and reports a device-detected wait timeout. */
int inferlab_cuda_peer_exchange_synchronize(InferlabCudaPeerExchange* exchange, void* stream,
                                            uint32_t timeout_ms, char* error, size_t error_capacity);

/* Closes the peers' buffers; every rank must have finished its exchanges. */
void inferlab_cuda_peer_exchange_destroy(InferlabCudaPeerExchange* exchange);

/*
 * The split-sequence decode and the exchange in ONE kernel: this rank decodes
 * its block range (the inferlab_cuda_paged_decode_partials arguments), and
 * the CTA that finishes each (sequence, kv-head) stores that kv-head's rows of
 * (m, l, o) into every rank's receive buffer of `exchange` (created with rows
 * = num_seqs * q_heads and the pool's head_dim), waits (bounded) for those
 * rows from all ranks and merges them in rank order into out [num_seqs *
 * q_heads][head_dim] - the same bits as partials + exchange_combine. Takes
 * one step of `exchange`, like inferlab_cuda_peer_exchange_combine; a rank
 * with no blocks of the sequence calls that instead with an empty block. A
 * call rejected with an error (argument checks, workspace size, batch size)
 * takes no step, so the ranks' later calls still pair up.
 * Needs the fast decode kernel's pool geometry, and at most half of the
 * GPU's resident decode CTAs may wait at once (num_seqs * kv_heads).
 */
int inferlab_cuda_paged_decode_exchange(InferlabCudaKvPool* pool, const float* queries,
                                        const int32_t* block_tables, uint32_t max_blocks,
                                        const int32_t* context_lens, uint32_t num_seqs,
                                        uint32_t q_heads, uint32_t max_context_len, void* workspace,
                                        size_t workspace_bytes, InferlabCudaPeerExchange* exchange,
                                        float* out, void* stream, char* error, size_t error_capacity);

/* Library version string, e.g. "inferlab-b200 0.1 sm_100a". */
const char* inferlab_cuda_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* INFERLAB_ATTENTION_H */
