/*
 * slimkv_b200 — C ABI of the B200 (sm_100a) SlimKV decode path.
 *
 * Plain pointers, element strides and sizes; no framework types.  All
 * tensors are device pointers unless stated otherwise; bf16 tensors are
 * passed as `const void*` (IEEE bfloat16 storage).  `stream` is a
 * `cudaStream_t` passed as `void*`.  Every entry point validates its
 * arguments on the host before launching anything and returns
 * SLIMKV_OK (0) or a positive SLIMKV_ERR_* code; nothing is launched on
 * error.  No entry point allocates device memory: callers pass any
 * workspace they need, sized by the matching *_workspace_size query, so the
 * calls can be captured in CUDA graphs.  Kernels that wait on TMA copies
 * give up after a bounded time, set bits in a per-device status word and
 * return; read it with slimkv_device_status().
 */
#ifndef SLIMKV_B200_H
#define SLIMKV_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SLIMKV_API __attribute__((visibility("default")))
#else
#define SLIMKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SLIMKV_OK 0
#define SLIMKV_ERR_INVALID_ARGUMENT 1
#define SLIMKV_ERR_UNSUPPORTED_SHAPE 2
#define SLIMKV_ERR_ALIGNMENT 3
#define SLIMKV_ERR_WORKSPACE 4
#define SLIMKV_ERR_CUDA 5
#define SLIMKV_ERR_TENSOR_MAP 6

/* Device status bits written by kernels (slimkv_device_status). */
#define SLIMKV_DEVICE_TIMEOUT 0x1u
#define SLIMKV_DEVICE_BAD_LENGTH 0x2u
/* A kernel found its dynamic shared memory less aligned than it needs and
 * returned without work. */
#define SLIMKV_DEVICE_MISALIGNED 0x4u

/* Library version as 10000*major + 100*minor + patch. */
SLIMKV_API int slimkv_version(void);

/* Human-readable text of the last host-side error on this thread. */
SLIMKV_API const char* slimkv_last_error(void);

/*
 * Read (and optionally clear) the device status word of the current device.
 * Synchronises the device.  Returns SLIMKV_OK or SLIMKV_ERR_CUDA.
 */
SLIMKV_API int slimkv_device_status(unsigned int* status, int clear);

/* ------------------------------------------------------------------------
 * Split-KV decode attention — drop-in for the reference extension
 * `slimkv_fa2_decode_320.forward(q, k, v, softmax_scale, causal=False,
 * num_splits=0, pack_q=True, cache_seqlens=None)`
 * (kernels/fa2_decode/binding.cpp:35-121, bound at 123-130).
 *
 * BSHD layouts with element strides {batch, seq, head}; the last dimension is
 * contiguous.  q [B, Q, H, D], k [B, N, Hkv, D], v [B, N, Hkv, Dv]; a batch
 * stride of 0 for k/v (one cache shared by every row) is allowed.  H % Hkv
 * == 0, Q in {1, 2}.  D, Dv <= 320 and multiples of 8.  Row strides must be
 * multiples of 8 elements and pointers 16-byte aligned (TMA).
 * out [B, Q, H, Dv] bf16, lse [B, H, Q] fp32 contiguous (natural log).
 * `causal` is bottom-right aligned.  Rows that see no key get zero output
 * and lse = +inf when `lse_masked_positive` (the reference extension's
 * convention) else -inf.  `cache_seqlens` (optional, int32 [B], device)
 * limits each row's keys.  `num_splits` 0 picks the split count.
 * ---------------------------------------------------------------------- */
typedef struct {
    const void* q;
    int64_t q_stride[3];
    const void* k;
    int64_t k_stride[3];
    const void* v;
    int64_t v_stride[3];
    void* out;
    int64_t out_stride[3];
    float* lse;
    const int32_t* cache_seqlens;
    int batch, queries, heads, kv_heads, keys, head_dim, value_dim;
    float scale;
    int causal;
    int num_splits;
    int lse_masked_positive;
    int out_fp32;   /* 1: `out` is fp32 (the fp32-accumulated result, no bf16 cast) */
} slimkv_attention_args;

SLIMKV_API size_t slimkv_attention_workspace_size(const slimkv_attention_args* args);
SLIMKV_API int slimkv_attention_forward(const slimkv_attention_args* args, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Allocation-free variant of slimkv_attention_forward.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory — for
 * example a host runtime that reaches this library only through an FFI that
 * hands over existing device buffers and has no CUDA allocator of its own, or
 * an engine that reserves all device memory up front and forbids later
 * allocations.  Same arguments, checks and results as
 * slimkv_attention_forward, but the split scratch comes from a fixed
 * 16 MiB array compiled into the library (every GPU that loads the library
 * holds one until the process exits); calls needing more scratch fail with
 * SLIMKV_ERR_WORKSPACE and an explanatory message.  Nothing here allocates.
 * The first call on a device looks up that device's copy of the array, so
 * make it before capturing a stream into a CUDA graph.  All calls on a device
 * share the one array and it keeps the previous call's contents (no call
 * depends on them): calls that can overlap on the GPU — concurrent streams
 * or threads — race on it, so issue them in order on one stream.
 * ---------------------------------------------------------------------- */
SLIMKV_API int slimkv_attention_forward_noalloc(const slimkv_attention_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Fused latent decode step — replaces steps 3-8 of the reference decode
 * `slimkv.llama3.fa2_decode.decode` (slimkv/llama3/fa2_decode.py:77-166):
 * BF16-exact RoPE of q and of the new raw key, cache append of the new raw
 * K/V and Beacon latents (llama3/memory.py:233-278, static_decode.py:156-171),
 * raw-branch grouped attention, q-absorb into Beacon-K latent space, latent
 * split-KV attention (causal on a Beacon-insertion row), V up-projection,
 * up-projection biases and the LSE merge.  Writes the attention output
 * [B, L, H*D] that feeds o_proj.
 *
 * Cache layout (per layer, this library's native HBM layout):
 *   raw_k_rot / raw_v : [B, raw_capacity, Hkv, D] bf16 token-major, strides
 *                       {raw_stride_batch, raw_stride_token} elements (head
 *                       stride D).  Rows 0..S-1 sinks, then the open window's
 *                       raw tail, then the current token.  raw_k_rot holds
 *                       keys already rotated at their compressed positions.
 *   raw_k_pre         : optional pre-RoPE copy of the keys (same layout).
 *   lat_k / lat_v     : [B, lat_capacity, Rk] / [B, lat_capacity, Rv] bf16,
 *                       strides {lat_stride_batch, lat_stride_row}; rows are
 *                       history latents then open-window latents.
 * Per-step metadata (int32 device arrays [B]):
 *   raw_len    : raw keys incl. the current token (its row is raw_len-1)
 *   latent_len : latents incl. a Beacon inserted this step (row latent_len-1)
 *   query_len  : 1, or 2 when this row inserts a Beacon (optional; NULL
 *                means `length` for every row)
 *   qpos       : [B, length] compressed positions of the queries
 * New entries this step (bf16, pre-RoPE): new_k / new_v [B, Hkv*D] from
 * k_proj/v_proj; new_lat_k [B, Rk] / new_lat_v [B, Rv] from the Beacon
 * down-projections (read only for rows whose query_len is 2).  Any of the
 * new_* pointers may be NULL to skip that append.
 * q [B, L, H, D] pre-RoPE (element strides {batch, seq, head}).
 * uk / uv: up-projection weights [Hkv*D, Rk] / [Hkv*D, Rv] (nn.Linear
 * weights), optional biases uk_bias / uv_bias [Hkv*D].
 * cos / sin: fp32 tables [rope_positions, D].
 * ---------------------------------------------------------------------- */
typedef struct {
    int batch, length, heads, kv_heads, head_dim, rank_k, rank_v;
    float scale;
    const void* q;
    int64_t q_stride[3];
    void* raw_k_rot;
    void* raw_v;
    void* raw_k_pre;
    int64_t raw_stride_batch, raw_stride_token;
    int raw_capacity;
    void* lat_k;
    void* lat_v;
    int64_t lat_stride_batch, lat_stride_row;
    int lat_capacity;
    const int32_t* raw_len;
    const int32_t* latent_len;
    const int32_t* query_len;
    const int32_t* qpos;
    const void* new_k;
    const void* new_v;
    int64_t new_stride;       /* elements between batch rows of new_k/new_v (0 = Hkv*D) */
    const void* new_lat_k;
    const void* new_lat_v;
    int64_t new_lat_stride;   /* elements between batch rows of new_lat_k/v (0 = R) */
    const void* uk;
    const void* uv;
    const void* uk_bias;
    const void* uv_bias;
    const float* cos;
    const float* sin;
    int rope_positions;
    void* out;
    int64_t out_stride[2];
    int out_fp32;   /* 1: `out` is fp32 (the fp32-accumulated result, no bf16 cast) */
    /* Host-side upper bounds of latent_len / raw_len used to plan the split
     * counts (0 = the capacities).  On the split-KV route a sequence longer
     * than the rows the plan covers is flagged SLIMKV_DEVICE_BAD_LENGTH (its
     * extra rows are not attended); the tensor-core route plans on the
     * device from the lengths themselves, up to the capacities. */
    int latent_len_max;
    int raw_len_max;
    /* Split counts (0 = chosen from the byte volume and the SM count).  On the
     * tensor-core route (32 query heads, ranks <= 320) the work is split on
     * the device instead: latent_splits then sets the number of persistent
     * CTAs of the launch and raw_splits the CTAs given to the raw branch. */
    int latent_splits;
    int raw_splits;
    /* Optional cudaEvent_t handles (NULL = none) recorded on `stream` right
     * before and after the attention launch (both branches), so a caller can
     * time that kernel alone.  Leave NULL inside CUDA graph capture. */
    void* attn_event_begin;
    void* attn_event_end;
    /* Paged latent cache (optional; NULL lat_pages = the dense lat_k / lat_v
     * above).  The vLLM plugin's Beacon pages (paged_cache.py:12-87): page p
     * at lat_pages + p * lat_page_stride (bf16 elements) holds
     * [lat_sink_elements][lat_slots x (rank_k + rank_v)]; latent row n of
     * sequence b is in page lat_table[b * lat_table_stride + n / lat_slots].
     * The attention reads the pages directly; the prologue appends the new
     * Beacon row there.  lat_slots must be a multiple of 16 and the
     * 32-query-head tensor-core route is required. */
    void* lat_pages;
    int64_t lat_page_stride;
    int lat_slots;
    int lat_sink_elements;
    const int32_t* lat_table;
    int64_t lat_table_stride;
    int lat_num_pages;
    /* Sequence split (optional): partial results of shards of one sequence's
     * keys, merged across GPUs afterwards with the LSE merge of
     * fa2_decode.py:57-66 taken over N parts.  out_lse (NULL = not written):
     * fp32 [B][L][H], the natural-log sum of exp of each output row's scores
     * over this call's keys (latent, with the K-bias shift, and raw); -inf for
     * a row that sees no key.  latent_shard != 0: this call's latent cache is
     * a shard that does not hold this step's Beacon row, so the latent branch
     * is not causal (new_lat_k / new_lat_v must be NULL). */
    float* out_lse;
    int latent_shard;
    /* Bound of every pipeline wait inside the attention kernel in ns (0 = 2 s).
     * A wait that runs out sets SLIMKV_DEVICE_TIMEOUT and the kernel returns
     * early; a short bound lets a caller (or a test) check that path. */
    uint64_t wait_limit_ns;
    /* Element stride between the KV heads of one token in raw_k_rot / raw_v /
     * raw_k_pre (0 = head_dim: the token-major layout above).  A head-major
     * cache [B, Hkv, raw_capacity, D] passes raw_stride_token = head_dim and
     * raw_stride_head = raw_capacity * head_dim. */
    int64_t raw_stride_head;
    /* The step's work plan from slimkv_decode_plan (int32 words on the
     * device), shared by the step's layers: the call then skips planning and
     * its attention launch starts while its prologue finishes (the tensor-core
     * route; ignored elsewhere).  NULL: the call plans in its workspace.  It
     * must have been computed from this call's raw_len / latent_len /
     * query_len values. */
    const int32_t* plan;
} slimkv_latent_decode_args;

SLIMKV_API size_t slimkv_latent_decode_workspace_size(const slimkv_latent_decode_args* args);
SLIMKV_API int slimkv_latent_decode(const slimkv_latent_decode_args* args, void* workspace,
                         size_t workspace_bytes, void* stream);

/* The work plan of a fused decode step (the split of the latent and raw rows
 * of every sequence over the attention CTAs), from the device lengths in
 * `args` (raw_len, latent_len, query_len and the shapes; other pointers are
 * not read).  Every layer of a step has the same lengths, so one plan serves
 * all of them (slimkv_latent_decode_args.plan); it replaces the planning that
 * each call otherwise does on its own.  `plan` holds slimkv_decode_plan_words
 * int32 words; on the split-KV route nothing is written and the plan is
 * ignored.  No counterpart in the reference: its decode has no batched
 * device schedule. */
SLIMKV_API size_t slimkv_decode_plan_words(const slimkv_latent_decode_args* args);
SLIMKV_API int slimkv_decode_plan(const slimkv_latent_decode_args* args, int32_t* plan, void* stream);

/* ------------------------------------------------------------------------
 * BF16-exact decode RoPE — drop-in for `decode_ops.fused_rope`
 * (slimkv/llama3/decode_ops.py:14-31, kernel decode_kernels.py:8-51).
 * q [B, H, Q, D] rotated at qpos [B, Q] (row stride qpos_stride); k
 * [B, Hkv, K, D] where key s < sink sits at position s, key s in
 * [sink, K-1) at raw_idx[s-sink] + sink + history and key K-1 at qpos[b][0].
 * Element strides {batch, head, seq}; outputs contiguous [B,H,Q,D] and
 * [B,Hkv,K,D].  raw_idx is int64 [K-1-sink] (may be NULL when K-1 == sink).
 * ---------------------------------------------------------------------- */
SLIMKV_API int slimkv_rope_decode(const void* q, const int64_t q_stride[3], const void* k,
                       const int64_t k_stride[3], const float* cos, const float* sin,
                       int rope_positions, const int64_t* qpos, int64_t qpos_stride,
                       const int64_t* raw_idx, int sink, int history, int batch, int heads,
                       int kv_heads, int queries, int keys, int head_dim, void* q_out,
                       void* k_out, void* stream);

/* ------------------------------------------------------------------------
 * BF16-exact RoPE of cache rows at per-sequence positions — the key half of
 * `decode_ops.fused_rope` (decode_kernels.py:8-51) for a batch whose
 * sequences sit at different positions (the vLLM plugin's requests, whose
 * raw tails are read from pages every step, paged_model.py:7-52):
 *   out[b, t, h, :] = rope(x[b, t, h, :]) at positions[b * positions_stride + t]
 * for t < counts[b] (counts NULL = all `tokens`), rounding to bf16 after each
 * multiply and after the add.  x / out bf16 with element strides {batch,
 * token, head} (last dim contiguous), distinct buffers; positions int32.
 * ---------------------------------------------------------------------- */
SLIMKV_API int slimkv_rope_rows(const void* x, const int64_t x_stride[3], void* out, const int64_t out_stride[3],
                                const int32_t* positions, int64_t positions_stride, const int32_t* counts,
                                int batch, int tokens, int heads, int head_dim, const float* cos, const float* sin,
                                int rope_positions, void* stream);

/* ------------------------------------------------------------------------
 * LSE merge — drop-in for `decode_ops.fused_merge`
 * (slimkv/llama3/decode_ops.py:34-48, kernel decode_kernels.py:54-76).
 * raw/latent [B, H, Q, D] bf16 (strides {batch, head, seq}), lse fp32
 * [B, H, Q] (strides {batch, head, seq}); out contiguous [B, H, Q, D] bf16.
 * ---------------------------------------------------------------------- */
/* ------------------------------------------------------------------------
 * Device-side decode schedule — the per-sequence form of the reference's
 * fast decode bookkeeping `LlamaMemory._step` (slimkv/llama3/memory.py:
 * 101-162) for an interleaved window of `window` raw tokens with one Beacon
 * after every `ratio` raw tokens (slimkv/memory.py:491-567).  One thread per
 * sequence reads its counters history[b] (completed-window latents) and
 * tail[b] (raw tokens already in the open window, T), writes this step's
 *   query_len[b]  = 1 + ((T + 1) % ratio == 0)        (Beacon inserted)
 *   raw_len[b]    = sink + T + 1
 *   latent_len[b] = history + T / ratio + (query_len - 1)
 *   qpos[b][0..1] = sink + history + T + T / ratio (+1 for the Beacon)
 * and advances T (closing the window, history += window / ratio, when
 * T + 1 == window).  All arrays int32 on the device; qpos is [B, 2].
 * ---------------------------------------------------------------------- */
SLIMKV_API int slimkv_decode_schedule(int batch, int sink, int window, int ratio, int32_t* history,
                                      int32_t* tail, int32_t* raw_len, int32_t* latent_len,
                                      int32_t* query_len, int32_t* qpos, void* stream);

SLIMKV_API int slimkv_merge(const void* raw, const int64_t raw_stride[3], const float* raw_lse,
                 const int64_t raw_lse_stride[3], const void* latent,
                 const int64_t latent_stride[3], const float* latent_lse,
                 const int64_t latent_lse_stride[3], int batch, int heads, int queries,
                 int head_dim, void* out, void* stream);

/* ------------------------------------------------------------------------
 * Paged cache IO in the vLLM plugin's page layouts, byte for byte
 * (slimkv/vllm_plugin/paged_cache.py:12-127).  Batched over sequences: row b
 * of `table` (int32, device, `table_stride` entries) is sequence b's block
 * table.  Copies are exact (bf16 bits).  A page id or position outside the
 * allocation sets SLIMKV_DEVICE_BAD_LENGTH and is skipped.
 * ---------------------------------------------------------------------- */
typedef struct {
    void* pages;              /* bf16, physical page p at pages + p * page_stride */
    int64_t page_stride;      /* elements between physical pages */
    int slots;                /* Beacon rows per page: raw_block_size / token_ratio */
    int rank_k, rank_v;       /* a row is K (rank_k) then V (rank_v) */
    int sink_elements;        /* 2 * raw_width: sink K then V at the page start */
    const int32_t* table;
    int64_t table_stride;
    int num_pages;            /* allocation size, for the bounds checks */
} slimkv_beacon_pages;

/* BeaconPages.append (paged_cache.py:78-87): rows [start[b], start[b]+count)
 * of sequence b <- key[b][i] (rank_k) ++ value[b][i] (rank_v). */
SLIMKV_API int slimkv_beacon_pages_append(const slimkv_beacon_pages* pages, int batch, const int32_t* start,
                                          int count, const void* key, int64_t key_stride_batch,
                                          int64_t key_stride_row, const void* value, int64_t value_stride_batch,
                                          int64_t value_stride_row, void* stream);
/* BeaconPages.read (paged_cache.py:64-76): the first count[b] rows of
 * sequence b -> dense key[b][i], value[b][i] (rows past count[b] untouched). */
SLIMKV_API int slimkv_beacon_pages_gather(const slimkv_beacon_pages* pages, int batch, const int32_t* count,
                                          int max_count, void* key, int64_t key_stride_batch,
                                          int64_t key_stride_row, void* value, int64_t value_stride_batch,
                                          int64_t value_stride_row, void* stream);
/* BeaconPages.write_sink / read_sink (paged_cache.py:89-100): the sink token
 * (key[b], value[b]: raw_width elements each) of sequence b at the start of
 * its root page table[b][0]; write = 1 stores, 0 loads. */
SLIMKV_API int slimkv_beacon_pages_sink(const slimkv_beacon_pages* pages, int batch, void* key, void* value,
                                        int64_t stride_batch, int write, void* stream);

typedef struct {
    void* pages;              /* bf16 [blocks][block_size][2 (K, V)][kv_heads][head_dim] */
    int block_size, kv_heads, head_dim;
    const int32_t* table;
    int64_t table_stride;
    int num_blocks;
} slimkv_raw_pages;

/* RawPages.write (paged_cache.py:117-127): absolute raw positions
 * [start[b], start[b]+count) of sequence b <- key/value [B][count][Hkv][D]. */
SLIMKV_API int slimkv_raw_pages_write(const slimkv_raw_pages* pages, int batch, const int32_t* start, int count,
                                      const void* key, int64_t key_stride_batch, int64_t key_stride_token,
                                      const void* value, int64_t value_stride_batch, int64_t value_stride_token,
                                      void* stream);
/* RawPages.read (paged_cache.py:108-115): count[b] tokens from start[b] ->
 * key/value [B][max_count][Hkv][D] (rows past count[b] untouched). */
SLIMKV_API int slimkv_raw_pages_read(const slimkv_raw_pages* pages, int batch, const int32_t* start,
                                     const int32_t* count, int max_count, void* key, int64_t key_stride_batch,
                                     int64_t key_stride_token, void* value, int64_t value_stride_batch,
                                     int64_t value_stride_token, void* stream);

/* ------------------------------------------------------------------------
 * Prefill window projection with Beacon roles and the cache append.
 *
 * Replaces, for one interleaved chunk of a prefill window,
 *   LlamaAttention.qkv_proj_with_beacon(hidden, beacon_size, beacon_indices,
 *       return_latents=True)            (slimkv/llama3/modeling_llama.py:1291-1345)
 *   LlamaAttention._incremental_cache   (modeling_llama.py:1347-1367)
 * under the prefill metadata of prefill_ops.prepare_metadata
 * (slimkv/llama3/prefill_ops.py:17-36: raw_indices / beacon_indices of the
 * chunk, no replica rows), and the cache writes that follow them:
 * Memory.update_memory (slimkv/llama3/memory.py:233-278) for dense caches
 * and flush_memory (slimkv/vllm_plugin/paged_model.py:55-83) for pages.
 *
 * Every row is projected by the ONE weight set its role selects (the
 * reference projects every row through both and selects with torch.where):
 *   raw row    i (chunk row raw_rows[i]):    q = h W_q^T (+b_q),
 *              k = h W_k^T (+b_k),  v = h W_v^T (+b_v)
 *   Beacon row j (chunk row beacon_rows[j]): q = h W_bq^T (+b_bq),
 *              lk = h W_kd^T,  lv = h W_vd^T  (latents, no bias),
 *              k = lk U_k^T (+b_uk),  v = lv U_v^T (+b_uv)
 * with fp32 accumulation and one rounding to bf16 per output (nn.Linear in
 * bf16).  k/v of Beacon rows are up-projected from the bf16 latents.
 * Weights are nn.Linear weights [out][in] (row-major bf16, rows 16-byte
 * aligned); biases are bf16 vectors or NULL.  W_kd and W_vd may be the same
 * pointer (shared K/V down-projection).
 *
 * Every output is optional (NULL = not computed):
 *   query/key/value  [B][rows][.] chunk rows (pre-RoPE), row r of sequence b
 *                    at base + b*stride_batch + r*stride_row;
 *   key_latent/value_latent  Beacon j at row (latent_start ? latent_start[b] : 0)
 *                    + j of latent_rows rows per sequence (a per-chunk
 *                    [B][beacon_count][R] buffer, or the dense latent cache
 *                    at its append cursor);
 *   beacon_pages     Beacon j at logical row beacon_start[b] + j (BeaconPages.append);
 *   raw_key_cache/raw_value_cache  dense [B][raw_cache_rows][kv_heads*head_dim]
 *                    raw cache: raw row i >= raw_first at row raw_start[b] + i;
 *   raw_pages        raw row i >= raw_first at absolute position raw_start[b] + i
 *                    (RawPages.write);
 *   write_sink != 0  the raw row at position raw_start[b] + i == 0 also goes
 *                    to the sink of beacon_pages' root page table[b][0]
 *                    (BeaconPages.write_sink).
 * key/value of Beacon rows need key_latent/value_latent (they are read back
 * by the up-projection).  Index lists are int32 device arrays shared by all
 * sequences; an index outside [0, rows), a cache row outside its buffer or a
 * page id outside the allocation sets SLIMKV_DEVICE_BAD_LENGTH and the row is
 * skipped.
 * ---------------------------------------------------------------------- */
typedef struct {
    int batch, rows, hidden;
    const void* hidden_states;                 /* bf16 [B][rows][hidden] */
    int64_t hidden_stride_batch, hidden_stride_row;
    const int32_t* raw_rows;                   /* metadata.raw_indices */
    int raw_count;
    const int32_t* beacon_rows;                /* metadata.beacon_indices */
    int beacon_count;
    int heads, kv_heads, head_dim, rank_k, rank_v;
    const void *w_q, *b_q, *w_k, *b_k, *w_v, *b_v;
    const void *w_bq, *b_bq, *w_k_down, *w_v_down, *w_k_up, *b_k_up, *w_v_up, *b_v_up;
    void* query;
    int64_t query_stride_batch, query_stride_row;
    void* key;
    int64_t key_stride_batch, key_stride_row;
    void* value;
    int64_t value_stride_batch, value_stride_row;
    void* key_latent;
    int64_t key_latent_stride_batch, key_latent_stride_row;
    void* value_latent;
    int64_t value_latent_stride_batch, value_latent_stride_row;
    int latent_rows;                           /* rows per sequence of key/value_latent (0: beacon_count) */
    const int32_t* latent_start;               /* [B] row of Beacon 0 in key/value_latent, or NULL */
    const slimkv_beacon_pages* beacon_pages;
    const int32_t* beacon_start;               /* [B] logical page row of Beacon 0 */
    const int32_t* raw_start;                  /* [B] raw position of raw row 0 */
    int raw_first;
    void* raw_key_cache;
    void* raw_value_cache;
    int64_t raw_cache_stride_batch, raw_cache_stride_row;
    int raw_cache_rows;                        /* rows per sequence of the dense raw cache */
    const slimkv_raw_pages* raw_pages;
    int write_sink;
    void* workspace;                           /* optional split-K scratch (16-byte aligned) */
    size_t workspace_bytes;
} slimkv_window_project_args;

/* Workspace for the split-K path (0 when the call does not split).  A call
 * whose output tiles do not fill the GPU splits each reduction into slices
 * that store fp32 partial tiles in the workspace; a second kernel sums them
 * in slice order (deterministic), adds the bias, rounds and stores.  Without
 * a large enough workspace the call runs unsplit (fewer CTAs; results may
 * differ from the split ones in the last bit).  Calls sharing a workspace
 * must be ordered (one stream). */
SLIMKV_API size_t slimkv_window_project_workspace_size(const slimkv_window_project_args* args);
SLIMKV_API int slimkv_window_project(const slimkv_window_project_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Prefill RoPE — drop-in for prefill_ops.fused_prefill_rope
 * (slimkv/llama3/prefill_ops.py:48-74, kernel prefill_kernels.py:7-53).
 * q [B][Hq][Q][D] and k [B][Hk][K][D] with element strides {batch, head,
 * seq} (last dim contiguous); outputs with their own strides.  Query s is
 * rotated at positions[b][K - Q + s], key s at positions[b][s] (int64, row
 * stride positions_stride).  Key s is a Beacon key (kept as is) when
 * s < prefix = K - role_count and s >= sink, or roles[s - prefix] is 1 or 2
 * (int64 roles).  Rotation is BF16-exact: out = bf16(bf16(x c) + bf16(r s))
 * with c, s the fp32 cos/sin table entries rounded to bf16 and r =
 * rotate_half(x).  cos/sin are fp32 [rope_positions][D].
 * ---------------------------------------------------------------------- */
SLIMKV_API int slimkv_prefill_rope(const void* q, const int64_t q_stride[3], const void* k,
                                   const int64_t k_stride[3], const float* cos, const float* sin,
                                   int rope_positions, const int64_t* positions, int64_t positions_stride,
                                   const int64_t* roles, int role_count, int sink, int batch, int heads,
                                   int kv_heads, int queries, int keys, int head_dim, void* q_out,
                                   const int64_t q_out_stride[3], void* k_out, const int64_t k_out_stride[3],
                                   void* stream);

/* ------------------------------------------------------------------------
 * Beacon K/V reconstruction for the reconstruct decode backend — replaces
 * ReconstructionCache.materialize (slimkv/llama3/memory.py:26-48) and the
 * per-step history up-projection of reconstruction_attention
 * (tools/benchmark/context_decode_runtime.py:298-344):
 *   key[b][start_b + r]   = bf16(lat_k[b][r] . w_k_up^T + b_k_up)     (Hkv*D)
 *   value[b][start_b + r] = bf16(lat_v[b][r] . w_v_up^T + b_v_up)
 * for r < rows (and r < row_count[b] when row_count, device int32 [B], is
 * given: the rows of a sequence past its latent count are neither read nor
 * written), start_b = out_start[b] (device int32 [B], NULL = 0), on the
 * tensor cores with fp32 accumulation and one rounding, as a bf16 nn.Linear.
 * lat_k / lat_v [B][lat_capacity][R] rows (element strides lat_stride_batch,
 * lat_stride_row; multiples of 8, 16-byte aligned); w_*_up [Hkv*D][R] as
 * nn.Linear weights; biases [Hkv*D] or NULL; key / value [B][out_rows][Hkv*D]
 * with element strides out_stride_batch / out_stride_row (multiples of 8).
 * A destination row past out_rows is skipped and flagged
 * SLIMKV_DEVICE_BAD_LENGTH.  workspace (optional) enables split-K for small
 * calls; size it with slimkv_reconstruct_kv_workspace_size.
 * ---------------------------------------------------------------------- */
typedef struct {
    int batch, rows, kv_heads, head_dim, rank_k, rank_v;
    const void* lat_k;
    const void* lat_v;
    int64_t lat_stride_batch, lat_stride_row;
    int lat_capacity;
    const void* w_k_up;
    const void* b_k_up;
    const void* w_v_up;
    const void* b_v_up;
    void* key;
    void* value;
    int64_t out_stride_batch, out_stride_row;
    int out_rows;
    const int32_t* out_start;
    void* workspace;
    size_t workspace_bytes;
    const int32_t* row_count;
} slimkv_reconstruct_args;

SLIMKV_API size_t slimkv_reconstruct_kv_workspace_size(const slimkv_reconstruct_args* args);
SLIMKV_API int slimkv_reconstruct_kv(const slimkv_reconstruct_args* args, void* stream);

/* ------------------------------------------------------------------------
 * N-part LSE merge of partial attention — the cross-GPU step of a sequence
 * split: merge_attention (slimkv/llama3/fa2_decode.py:57-66), which merges two
 * partitions of one row's keys, generalised to N partitions:
 *   T = log sum_i exp(lse_i),  out = sum_i exp(lse_i - T) part_i.
 * part_out: fp32, part i of row r at part_out + i*part_stride + r*dim;
 * part_lse: fp32, lse of part i of row r at part_lse + i*lse_part_stride + r
 * (natural log, -inf for a part without keys).  The layout matches one
 * all-gather of per-rank [rows*dim outputs | rows lses] buffers.  out
 * [rows][dim] bf16, or fp32 when out_fp32; out_lse [rows] fp32 (nullable).
 * Rows without keys in any part get zero output and lse -inf.  dim a multiple
 * of 4, part_stride a multiple of 4, 16-byte aligned part_out (and out when
 * fp32; 8-byte when bf16).
 * ---------------------------------------------------------------------- */
typedef struct {
    int parts, rows, dim;
    const float* part_out;
    int64_t part_stride;
    const float* part_lse;
    int64_t lse_part_stride;
    void* out;
    int out_fp32;
    float* out_lse;
} slimkv_merge_partials_args;

SLIMKV_API int slimkv_merge_partials(const slimkv_merge_partials_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Prefill attention (tcgen05 flash attention forward) — the attention of a
 * prefill chunk when the history stays in latent form, replacing the
 * materialisation of every history latent (ReconstructionCache.materialize,
 * slimkv/llama3/memory.py:26-48, joined at modeling_llama.py:1650-1681)
 * followed by one flash attention.  One call attends one part:
 *   out[b, t, g*R + j, :] = softmax_k(scale q[b, t, g*R + j, :] . k[b, k, g, :]) v[b, k, g, :]
 * over keys k < kv_len[b] (and k <= causal_offset + t when causal), R =
 * rows_per_token query heads per KV head g.  The history part passes the
 * queries absorbed into latent space with every head of the chunk as rows
 * of the one latent head (kv_heads 1, R = H) and the latents as k / v; the
 * chunk part passes the rotated queries, keys and values of the sinks and
 * the chunk (causal, bottom-right: causal_offset = keys before the chunk).
 * q [B][tokens][kv_heads*R][dim_qk], k [B][kv_capacity][kv_heads][dim_qk],
 * v likewise with dim_v: bf16, element strides {batch, token, head}
 * (multiples of 8, last dimension contiguous, 16-byte aligned); out bf16
 * [B][tokens][heads][dim_v] strides out_stride; lse fp32 natural log at
 * lse[b*lse_stride[0] + t*lse_stride[1] + head] (nullable; -inf for a row
 * without keys).  dims multiples of 8 up to 320; R at most 128.
 * ---------------------------------------------------------------------- */
typedef struct {
    int batch, kv_heads, rows_per_token, tokens;
    int dim_qk, dim_v;
    const void* q;
    int64_t q_stride[3];
    const void* k;
    const void* v;
    int64_t kv_stride[3];
    int kv_capacity;
    const int32_t* kv_len;
    int causal, causal_offset;
    float scale;
    void* out;
    int64_t out_stride[3];
    float* lse;
    int64_t lse_stride[2];
    uint64_t wait_limit_ns;    /* bound of every pipeline wait (0: 2 s) */
} slimkv_prefill_attention_args;

SLIMKV_API int slimkv_prefill_attention(const slimkv_prefill_attention_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Decoder-layer element-wise steps of the batched decode runtime.
 * slimkv_rms_norm replaces LlamaRMSNorm.forward (slimkv/llama3/
 * modeling_llama.py:79-95): out = weight * bf16(x * rsqrt(mean(x^2) + eps)),
 * the mean in fp32, bf16 rows x / out with row strides in elements, weight
 * [hidden] bf16; hidden a multiple of 8, at most 8192; 16-byte aligned rows.
 * slimkv_silu_mul replaces act_fn(gate_proj(x)) * up_proj(x) of
 * LlamaMLP.forward (modeling_llama.py:97-113) with the two projections as
 * one row [gate (intermediate) | up (intermediate)]: out = bf16(silu(gate))
 * * up, rounded to bf16; intermediate a multiple of 8, 16-byte aligned rows.
 * ---------------------------------------------------------------------- */
SLIMKV_API int slimkv_rms_norm(const void* x, int64_t x_row_stride, const void* weight, void* out,
                               int64_t out_row_stride, int rows, int hidden, float eps, void* stream);
SLIMKV_API int slimkv_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out, int64_t out_row_stride,
                               int rows, int intermediate, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SLIMKV_B200_H */
