/* beam_b200.h -- C ABI of the B200 beam-decode path.
 *
 * Plain pointers and sizes only.  Device pointers are CUDA global-memory
 * addresses on the current device; `stream` is a cudaStream_t passed as
 * void* (NULL = legacy default stream).  Every call returns a be_status;
 * be_last_error() gives the text of the last failure on the calling thread.
 * Kernels never trap: an out-of-range page id or slot found on the device is
 * skipped and recorded in a device status word (be_device_status()).
 *
 * Each entry point cites the reference interface it replaces
 * (brian030128/beam_engine, paths relative to the project root).
 */
#ifndef BEAM_B200_H
#define BEAM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  BE_OK = 0,
  BE_EINVAL = 1,           /* bad argument (-> ValueError)                      */
  BE_ENOMEM = 2,           /* page pool exhausted (-> MemoryError, page_table.py:87-88) */
  BE_ECUDA = 3,            /* CUDA runtime error                               */
  BE_ENOT_ALLOCATED = 4,   /* free of a page that is not allocated (a warning, page_table.py:117-119) */
  BE_ECAPACITY = 5,        /* caller buffer too small; required size reported   */
  BE_EDEVICE_RANGE = 6,    /* device status: an index was out of range and skipped */
  BE_EDEVICE_TIMEOUT = 7,  /* device status: a bounded pipeline wait expired; output invalid */
  BE_ENOTSUP = 8           /* plan shape this path does not serve (the caller takes another) */
} be_status;

typedef enum { BE_F32 = 0, BE_F16 = 1, BE_BF16 = 2 } be_dtype;

const char* be_last_error(void);
int be_version(void);

/* Device status word (per device).  be_device_status copies it to *out
 * (synchronous on `stream`), be_device_status_clear resets it to 0.        */
int be_device_status(int* out, void* stream);
int be_device_status_clear(void* stream);

/* ------------------------------------------------------------------------
 * Paged KV pool layout: per layer [num_pages, 2, page_size, num_kv_heads,
 * head_dim] (plane 0 = K, plane 1 = V), the reference's NHD pool
 * (src/beam_engine/page_table.py:62-72).  Several layers may be addressed in
 * one call through `pool_layer_stride` (elements between consecutive layers'
 * pools; the reference keeps one tensor per layer).
 * ---------------------------------------------------------------------- */

/* Replaces flashinfer.page.append_paged_kv_cache as called by
 * PageTable.write_blocks_vectorized (src/beam_engine/page_table.py:199-209).
 * Entry i (0 <= i < nnz) writes key/value row i into page
 * kv_indices[kv_indptr[batch_indices[i]] + positions[i] / page_size] at in-page
 * slot positions[i] % page_size, for layers 0..num_layers-1.
 * append_key/append_value: [num_layers][nnz][num_kv_heads][head_dim] with
 * `row_stride` elements between rows i and i+1 (head/dim contiguous) and
 * `input_layer_stride` elements between layers (so K/V can be read in place
 * from a fused QKV projection output).                                        */
int be_append_paged_kv(const void* append_key, const void* append_value, int64_t row_stride,
                       int64_t input_layer_stride, const int32_t* batch_indices,
                       const int32_t* positions, const int32_t* kv_indices, const int32_t* kv_indptr,
                       int nnz, void* paged_kv_cache, int64_t pool_layer_stride, int num_layers,
                       int num_pages, int page_size, int num_kv_heads, int head_dim, int dtype,
                       void* stream);

/* Copy-on-write fork of partially filled tail pages, all layers in one launch.
 * Replaces the per-layer copy loop of PageTable.copy_block
 * (src/beam_engine/page_table.py:96-106) issued by BeamState.add_filtered_results
 * (src/beam_engine/beam_state.py:190-191).  Copy j moves tokens [0, lens[j]) of K
 * and V from page src_pages[j] to page dst_pages[j] in every layer.  Copies must
 * not read a page another copy of the same call writes (true for one fork step:
 * sources are live leaves, destinations fresh pages).                         */
int be_fork_tail_copy(void* paged_kv_cache, int64_t pool_layer_stride, int num_layers,
                      int num_pages, int page_size, int num_kv_heads, int head_dim, int dtype,
                      const int32_t* src_pages, const int32_t* dst_pages, const int32_t* lens,
                      int num_copies, void* stream);

/* be_fork_tail_copy with the copy list in device memory, for a decode step
 * recorded once as a CUDA graph: copy_list = [count | src_pages[cap] |
 * dst_pages[cap] | lens[cap]] (int32).  The launch shape depends only on
 * num_sms, so the same recorded launch serves every step's list.            */
int be_fork_tail_copy_list(void* paged_kv_cache, int64_t pool_layer_stride, int num_layers,
                           int num_pages, int page_size, int num_kv_heads, int head_dim,
                           int dtype, const int32_t* copy_list, int cap, int num_sms,
                           void* stream);

/* ------------------------------------------------------------------------
 * Paged attention plans.  A plan is a flat int32 buffer built on the host by
 * be_cascade_plan / be_tree_plan, copied to the device by the caller, and run
 * by be_attn_run.  It lists work items, each "some queries of one group x a
 * token range of that group's KV", plus the per-query list of partial states
 * that be_attn_run merges by log-sum-exp.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t q_off;     /* first entry in the query list                          */
  int32_t q_len;     /* number of queries (rows = q_len * group size)          */
  int32_t kv_off;    /* first entry in the KV list (page ids or slot ids)      */
  int32_t kv_begin;  /* token range [kv_begin, kv_end) of the group's sequence */
  int32_t kv_end;
  int32_t kv_total;  /* group's full KV length (causal alignment)              */
  int32_t part_base; /* partial row of query 0 (>= 0) or -1: write output directly */
  int32_t flags;     /* BE_WORK_CAUSAL | BE_WORK_SLOTS                         */
} be_attn_work;

/* Every plan buffer starts with a copy of its be_attn_plan_info, padded to
 * BE_PLAN_HEADER_INTS ints, so kernels can read the counts on the device. */
#define BE_PLAN_HEADER_INTS 32

/* Longest wide (shared-prefix) work item the tensor-core kernel takes; the
 * cascade planner cuts decode-time prefix chunks to this length. */
#define BE_UMMA_MAX_TOKENS 128

#define BE_WORK_CAUSAL 1 /* query i sees tokens t < kv_total - q_len + i + 1 */
#define BE_WORK_SLOTS 2  /* KV list holds slot ids (page*page_size+i), else page ids */

typedef struct {
  int32_t n_work;        /* work items                                         */
  int32_t n_work_wide;   /* leading items whose rows exceed 16 (wide tiles)    */
  int32_t n_queries;     /* rows of q / out                                    */
  int32_t n_parts;       /* partial states (rows of mid_o / mid_lse)           */
  int32_t n_merge;       /* queries with >= 1 partial (merged by be_attn_run)  */
  int32_t off_work;      /* int32 offsets into the plan buffer                 */
  int32_t off_qlist;
  int32_t off_kvlist;
  int32_t off_merge_q;   /* [n_merge] query ids                                */
  int32_t off_merge_ptr; /* [n_merge + 1] CSR into merge_parts                 */
  int32_t off_merge_parts;
  int32_t total_ints;    /* ints to copy to the device                         */
  int32_t page_size;
  int32_t group_size;    /* num_qo_heads / num_kv_heads                        */
  int32_t any_slots;     /* some item lists slot ids (BE_WORK_SLOTS)           */
  int32_t max_item_tokens; /* longest work item (tokens)                      */
  int32_t total_tokens;  /* sum of work-item token ranges                      */
  int32_t max_wide_tokens; /* longest wide (> 16-row) work item (tokens)      */
} be_attn_plan_info;

/* Plans MultiLevelCascadeAttentionWrapper.plan + .run
 * (src/beam_engine/models/modeling_llama.py:733-755, :362; FlashInfer
 * cascade semantics: level l group g owns queries qo_indptr[l][g]..[g+1] and
 * pages kv_indices[l][kv_indptr[l][g]..[g+1]], kv_len =
 * (npages-1)*page_size + last_page_len[l][g]; only the last level is causal
 * when causal_last != 0; levels merged by LSE).  Arrays are host int32.
 * split_tokens = 0 picks the KV split per group from num_sms; > 0 forces it
 * (rounded to pages).  On BE_ECAPACITY info->total_ints holds the size needed. */
int be_cascade_plan(int num_levels, const int32_t* const* qo_indptr,
                    const int32_t* const* kv_indptr, const int32_t* const* kv_indices,
                    const int32_t* const* last_page_len, const int32_t* num_groups,
                    int num_queries, int page_size, int num_qo_heads, int num_kv_heads,
                    int causal_last, int split_tokens, int num_sms, int32_t* plan,
                    int64_t plan_capacity, be_attn_plan_info* info);

/* Plans fasttree_decode (src/beam_engine/attention/fasttree/kernel.py:288-348)
 * from the vnode metadata of prepare_fasttree_metadata_for_paged_cache
 * (attention/fasttree/preparation.py:11-225): vnode v attends queries
 * q_entries[q_offs[v] .. +q_lens[v]] to slots kv_entries[kv_offs[v] .. +kv_lens[v]];
 * request b merges the partial rows req_to_vnode_entries[r2v_offs[b] .. +r2v_lens[b]].
 * The KV entries themselves stay in the caller's device buffer (kv_entries_dev
 * is passed to be_attn_run as kv_list_override).                              */
int be_tree_plan(int num_vnodes, const int32_t* q_entries, int num_q_entries,
                 const int32_t* q_offs, const int32_t* q_lens, const int32_t* kv_offs,
                 const int32_t* kv_lens, const int32_t* r2v_entries, const int32_t* r2v_offs,
                 const int32_t* r2v_lens, int batch_size, int page_size, int num_qo_heads,
                 int num_kv_heads, int32_t* plan, int64_t plan_capacity, be_attn_plan_info* info);

/* The FastTree vnodes of be_fasttree_prepare as a page-list plan for the
 * tensor-core kernels (be_attn_run / be_attn_run_fixed without slot lists):
 * slots = the slot table the vnodes' kv_offs index (page * page_size + i).
 * Every vnode must cover whole pages from slot 0 (true of beam-trie trees:
 * nodes start at slot 0 of their page, non-leaf nodes are full); otherwise
 * BE_EINVAL and the caller keeps the slot-list plan of be_tree_plan.  Same attention as be_tree_plan,
 * split for the decode kernels like be_cascade_plan.                         */
int be_tree_plan_pages(int num_vnodes, const int32_t* q_entries, int num_q_entries,
                       const int32_t* q_offs, const int32_t* q_lens, const int32_t* kv_offs,
                       const int32_t* kv_lens, const int32_t* slots, int64_t num_slots,
                       int batch_size, int page_size, int num_qo_heads, int num_kv_heads,
                       int num_sms, int32_t* plan, int64_t plan_capacity,
                       be_attn_plan_info* info);

/* Runs a plan for one layer.  q: [n_queries][num_qo_heads][head_dim] with
 * q_row_stride elements between queries; paged_kv_cache: one layer's pool;
 * out: [n_queries][num_qo_heads][head_dim] (out_row_stride); lse (nullable):
 * [n_queries][num_qo_heads] float32, natural log.  mid_o / mid_lse: float32
 * scratch of n_parts*num_qo_heads*head_dim and n_parts*num_qo_heads floats.
 * kv_list_override (nullable): device int32 KV list used instead of the plan's.
 * Queries that appear in no work item get out = 0, lse = -inf.               */
int be_attn_run(const int32_t* plan_dev, const be_attn_plan_info* info, const void* q,
                int64_t q_row_stride, const void* paged_kv_cache, int num_pages,
                int num_qo_heads, int num_kv_heads, int head_dim, int dtype, float sm_scale,
                void* out, int64_t out_row_stride, float* lse, float* mid_o, float* mid_lse,
                const int32_t* kv_list_override, void* stream);

/* be_attn_run for callers that cannot allocate device memory.  No counterpart
 * in the reference (which always lets FlashInfer use a caller workspace).
 * Same arguments as be_attn_run minus mid_o / mid_lse: the partial rows go to
 * an array compiled into this library, BE_NOALLOC_SCRATCH_BYTES per device,
 * reserved on every GPU that loads the library until the process exits.
 *   - Plans needing more partial-row space (n_parts * Hq * (D + 1) * 4 bytes,
 *     roughly) fail with BE_ECAPACITY and a message; nothing is allocated.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - All calls share the one array: calls whose work overlaps on the GPU
 *     (different streams, or devices sharing a context) race and corrupt each
 *     other's results; serialise them.                                        */
#define BE_NOALLOC_SCRATCH_BYTES (16u << 20)
int be_attn_run_noalloc(const int32_t* plan_dev, const be_attn_plan_info* info, const void* q,
                        int64_t q_row_stride, const void* paged_kv_cache, int num_pages,
                        int num_qo_heads, int num_kv_heads, int head_dim, int dtype, float sm_scale,
                        void* out, int64_t out_row_stride, float* lse,
                        const int32_t* kv_list_override, void* stream);

/* Grid capacities of be_attn_run_fixed.  The launch configuration depends on
 * these only, so the call can be recorded once (e.g. in a CUDA graph) and
 * replayed with any plan that fits: the kernels read the plan's real counts
 * from its device-side header and idle the surplus CTAs.                     */
typedef struct {
  int32_t max_work;   /* >= n_work of every plan run this way                  */
  int32_t max_wide;   /* >= n_work_wide                                         */
  int32_t max_merge;  /* >= n_merge                                             */
  int32_t cluster;    /* CTAs per work item for narrow tiles (1..8)             */
  int32_t flags;      /* BE_CAPS_SLOTS: the plans hold slot lists (tree plans)   */
} be_attn_caps;
#define BE_CAPS_SLOTS 1

/* be_attn_run with a launch shape fixed by `caps` instead of a host-side plan
 * description: the plan at plan_dev (header included) may change between
 * calls without any host involvement.  Page-list plans with page size 16 use
 * the tensor-core kernels; wide items must span <= 256 tokens (the planner's
 * decode chunks do); a plan that breaks the caps is flagged in the device
 * status and its surplus items are skipped.  The plan must be in device
 * memory before the kernel preceding this call on the stream starts (a host
 * copy, as in a recorded decode step): the kernels read it while that kernel
 * finishes.  Same contract as MultiLevelCascadeAttentionWrapper.run
 * (modeling_llama.py:362).                                                   */
int be_attn_run_fixed(const int32_t* plan_dev, const be_attn_caps* caps, int page_size,
                      const void* q, int64_t q_row_stride, const void* paged_kv_cache,
                      int num_pages, int num_qo_heads, int num_kv_heads, int head_dim, int dtype,
                      float sm_scale, void* out, int64_t out_row_stride, float* lse,
                      float* mid_o, float* mid_lse, const int32_t* kv_list_override,
                      void* stream);

/* be_attn_run_fixed with the narrow (per-beam suffix) tiles on a second
 * stream: they start as soon as SMs free up from the shared-prefix tiles
 * instead of after them; the LSE merge waits for both on `stream`.  Both
 * streams must belong to the current device; inside a stream capture the
 * fork and join become graph dependencies.  side_stream NULL = one stream.  */
int be_attn_run_fixed_2s(const int32_t* plan_dev, const be_attn_caps* caps, int page_size,
                         const void* q, int64_t q_row_stride, const void* paged_kv_cache,
                         int num_pages, int num_qo_heads, int num_kv_heads, int head_dim,
                         int dtype, float sm_scale, void* out, int64_t out_row_stride, float* lse,
                         float* mid_o, float* mid_lse, const int32_t* kv_list_override,
                         void* stream, void* side_stream);

/* ------------------------------------------------------------------------
 * Beam-tile decode attention (the default decode path for 2-byte pools with
 * head_dim 128 and page size 16).  Same attention as be_cascade_plan +
 * be_attn_run -- MultiLevelCascadeAttentionWrapper.plan / .run
 * (modeling_llama.py:733-755, :362) -- in another plan form:
 *   - a tile is a run of consecutive queries (one prompt's beams, cut at the
 *     level-0 groups) of at most tile_rows query-head rows;
 *   - an entry is one page a tile reads: (page id, valid tokens from slot 0,
 *     query range [q_lo, q_hi) relative to the tile).  Every level-l group
 *     contributes one entry per page and per tile its query range overlaps;
 *     the last page has last_page_len tokens, the others page_size.  A page
 *     listed at two levels is attended twice, as the reference's cascade does;
 *   - a piece is a range of one tile's entries; one CTA per (piece, KV head)
 *     streams the pages through shared memory (TMA) into tcgen05 tiles
 *     (S = Q K^T, O = P V in TMEM, online softmax).  A tile of several pieces
 *     leaves partial rows that a second kernel, launched right after, merges
 *     by log-sum-exp.
 * Decode only: a causal last level whose groups hold more than one query
 * (a prompt) returns BE_ENOTSUP, and the caller plans with be_cascade_plan.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t n_tiles, n_pieces, n_entries, n_queries;
  int32_t off_tiles, off_pieces, off_entries, total_ints;
  int32_t page_size, group_size, tile_rows, n_part_pieces; /* pieces with partial rows */
  int32_t total_tokens;     /* sum of the entries' valid tokens                   */
  int32_t max_piece_entries;
  int32_t cluster;          /* > 1: every tile has exactly `cluster` pieces, merged in
                               the kernel through distributed shared memory        */
  int32_t pad1;
} be_tile_plan_info;
typedef struct {
  int32_t q_begin, q_len;   /* queries [q_begin, q_begin + q_len), rows = q_len * g */
  int32_t piece_begin, n_pieces;
  int32_t part_base;        /* first partial slot of the tile's pieces, -1 if one piece */
  int32_t pad0, pad1, pad2;
} be_attn_tile;
typedef struct { int32_t page, ntok, q_lo, q_hi; } be_attn_entry;
typedef struct {
  int32_t tile, ent_begin, ent_end, index;   /* entries [ent_begin, ent_end) of `tile` */
  int32_t q_begin, q_len, n_pieces, part_base; /* copies of the tile's fields          */
  be_attn_entry first[4];                      /* copies of the piece's first entries  */
} be_attn_piece;
/* Plan buffer: header (be_tile_plan_info, BE_PLAN_HEADER_INTS ints), pieces
 * (from off_pieces == BE_PLAN_HEADER_INTS), tiles, entries.                  */

/* Cascade levels (the arrays of be_cascade_plan) -> tile plan.  tile_rows is
 * 64 or 128.  cluster <= 1: about target_pieces pieces in all (~2 x SMs /
 * num_kv_heads), partial rows merged by a second kernel.  cluster in 2..16:
 * exactly `cluster` pieces per tile (some may be empty), run as one thread-
 * block cluster per (tile, KV head) that merges its partial rows through
 * distributed shared memory (no partial rows in global memory).  cluster -1:
 * chosen from target_pieces and the tile count (info->cluster reports it; 0 =
 * no cluster).  On BE_ECAPACITY info->total_ints holds the size needed.      */
int be_tile_plan(int num_levels, const int32_t* const* qo_indptr, const int32_t* const* kv_indptr,
                 const int32_t* const* kv_indices, const int32_t* const* last_page_len,
                 const int32_t* num_groups, int num_queries, int page_size, int num_qo_heads,
                 int num_kv_heads, int causal_last, int tile_rows, int target_pieces,
                 int cluster, int32_t* plan, int64_t plan_capacity, be_tile_plan_info* info);

/* Runs a tile plan in device memory (header included) on `stream`: the tile
 * kernel, and for plans made with cluster <= 1 the merge kernel.  The grid is
 * (max_pieces, num_kv_heads), clusters of `cluster` CTAs along x when
 * cluster > 1 (max_pieces a multiple of it; the plan must have been made with
 * the same cluster).  CTAs past the plan's piece count exit, so a recorded
 * launch serves every plan with n_pieces <= max_pieces, n_tiles <= max_tiles
 * and n_part_pieces <= max_part_pieces.  Every CTA reads its piece record
 * before the piece count, so the plan buffer must hold at least
 * BE_PLAN_HEADER_INTS + 24 * max_pieces ints.
 * part_o: [max_part_pieces][num_kv_heads][tile_rows][head_dim] elements of
 * `dtype` (partial rows are normalised, O / l) and
 * part_lse: [max_part_pieces][num_kv_heads][tile_rows] fp32 scratch (unused
 * with clusters; calls that share them must not overlap on the GPU).
 * lse (optional): natural-log LSE per (query, qo head).  plan_early != 0: the
 * plan is in device memory before the kernel preceding this call starts
 * (read before the programmatic-launch wait).                                */
int be_attn_tiles_run(const int32_t* plan_dev, int max_pieces, int max_tiles, int max_part_pieces,
                      int tile_rows, int page_size, const void* q, int64_t q_row_stride,
                      const void* paged_kv_cache, int num_pages, int num_qo_heads,
                      int num_kv_heads, int head_dim, int dtype, float sm_scale, void* out,
                      int64_t out_row_stride, float* lse, void* part_o, float* part_lse,
                      int cluster, int plan_early, void* stream);

/* ------------------------------------------------------------------------
 * Decoder-layer kernels of the model runner (the reference runs these as
 * separate PyTorch ops inside src/beam_engine/models/modeling_llama.py).
 * ---------------------------------------------------------------------- */

/* LlamaDecoderLayer residual add + LlamaRMSNorm (modeling_llama.py:68-86,
 * 577-621) in one pass: residual += delta (delta may be NULL), then
 * out = weight * cast(residual * rsqrt(mean(residual^2) + eps)).            */
int be_add_rmsnorm(void* residual, const void* delta, const void* weight, void* out, int rows,
                   int hidden, float eps, int dtype, void* stream);

/* RoPE (HF rotate_half, modeling_llama.py:113-157) on the q and k heads of a
 * fused QKV projection row [q heads | k heads | v heads] (row_stride elements
 * apart), q rotated in place, rotated k and v appended into page
 * write_page[i] slot write_pos[i] -- apply_rotary_pos_emb followed by
 * PageTable.write_blocks_vectorized (modeling_llama.py:464-514) in one launch.
 * inv_freq: [head_dim/2] float32 device array.  rope_k_in_place != 0 also
 * leaves the rotated k in the QKV row.                                       */
int be_rope_qkv_append(void* qkv, int64_t row_stride, int n, int num_qo_heads, int num_kv_heads,
                       int head_dim, const int32_t* positions, const float* inv_freq,
                       void* paged_kv_cache, int num_pages, int page_size,
                       const int32_t* write_page, const int32_t* write_pos, int rope_k_in_place,
                       int dtype, void* stream);

/* LlamaMLP activation (modeling_llama.py:160-173): out = silu(gate) * up on a
 * fused [n][2*ffn] gate|up projection.                                       */
int be_silu_mul(const void* gate_up, void* out, int n, int ffn, int dtype, void* stream);

/* Beam scoring (beam.py:266-317: logits / temperature -> log_softmax ->
 * topk(k)) in one launch.  logits [rows][ld] f32, first v columns used.
 * full_vocab != 0: out_val[rows][k] = log-probabilities of the k largest,
 * out_idx = vocab_offset + column (order: value desc, then id asc).
 * full_vocab == 0 (a vocabulary slice under tensor parallelism): out_val =
 * the slice's k largest scaled logits, row_max / row_sumexp = the slice's
 * max and sum(exp(x - max)) for a cross-rank log-sum-exp.  k <= 64.         */
int be_logsoftmax_topk(const float* logits, int64_t ld, int rows, int v, float temperature,
                       int k, int64_t vocab_offset, int full_vocab, float* out_val,
                       int64_t* out_idx, float* row_max, float* row_sumexp, void* stream);

/* Decode projection GEMM (the q/k/v, o, gate/up, down and lm_head matmuls of
 * LlamaAttention / LlamaMLP, modeling_llama.py:428-562, 577-621, which the
 * reference runs as torch linears): Y[T][N] = X[T][K] * W[N][K]^T, bf16
 * operands, fp32 accumulate, Y bf16 (out_dtype BE_BF16) or f32.  T <= 128,
 * N >= 128, K % 64 == 0, row strides ldx / ldw multiples of 8 elements.
 * split_k 0 = automatic (about two CTAs per SM); split-K partials go to
 * `workspace` (splits * T * N floats; a smaller workspace lowers the split). */
int be_gemm_tn(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
               int T, int N, int K, int out_dtype, int split_k, float* workspace,
               int64_t workspace_floats, void* stream);

/* The same GEMM through cuBLASLt: the first call of a shape outside stream
 * capture times cuBLASLt's top heuristic candidates on `stream` and keeps the
 * fastest (later calls and captured calls reuse it).  workspace: device
 * scratch of workspace_bytes for split-K algorithms.                        */
int be_gemm_lt(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
               int T, int N, int K, int out_dtype, void* workspace, int64_t workspace_bytes,
               void* stream);

/* ------------------------------------------------------------------------
 * Host page manager (no CUDA): FIFO page allocator + beam trie.  One
 * be_trie backs one PageTable and the BeamState objects over it.
 * Single-threaded, like the reference.
 * ---------------------------------------------------------------------- */
typedef struct be_trie be_trie;

/* PageTable.__init__ free list (src/beam_engine/page_table.py:59-60).       */
be_trie* be_trie_create(int page_size, int max_num_pages);
void be_trie_destroy(be_trie* t);
/* PageTable.allocate_block (page_table.py:77-94): pops the FRONT of the free
 * list; BE_ENOMEM when empty.                                               */
int be_alloc_page(be_trie* t, int32_t* page);
/* PageTable.free_block (page_table.py:110-124): appends to the BACK;
 * BE_ENOT_ALLOCATED (a warning, no state change) for a page not allocated.  */
int be_free_page(be_trie* t, int32_t page);
int be_num_free_pages(be_trie* t);
int be_is_allocated(be_trie* t, int32_t page);
/* Free list in FIFO order (up to cap entries); returns its length.          */
int be_free_list(be_trie* t, int32_t* out, int cap);
int64_t be_trie_warnings(be_trie* t);
int be_trie_num_nodes(be_trie* t);

/* TrieNode(tokens, page_id, parent) (src/beam_engine/beam_state.py:20-27);
 * parent = -1 for a root.  Node ids are stable handles.                      */
int be_node_new(be_trie* t, int32_t parent, int32_t page, const int32_t* tokens, int n,
                int32_t* node_out);
int be_node_info(be_trie* t, int32_t node, int32_t* parent, int32_t* page, int32_t* ntokens,
                 int32_t* nchildren);
int be_node_tokens(be_trie* t, int32_t node, int32_t* out, int cap);
int be_node_children(be_trie* t, int32_t node, int32_t* out, int cap);
int be_node_append_token(be_trie* t, int32_t node, int32_t token);
/* Root-to-leaf token sequence (beam_state.py:667-671); returns its length.  */
int64_t be_node_sequence(be_trie* t, int32_t leaf, int32_t* out, int64_t cap);

/* Token sequences of n leaves as CSR (DiverseBeamSearchStrategy._get_sequence_from_node,
 * src/beam_engine/beam_strategy.py:96-103: the walk up stops at a node with no
 * tokens).  seq_ptr [n + 1]; seq_tokens written up to cap; returns the total
 * length (-1 for an unknown leaf).                                           */
int64_t be_leaf_sequences(be_trie* t, int n, const int32_t* leaves, int32_t* seq_ptr,
                          int32_t* seq_tokens, int64_t cap);
/* BeamState.add_root_sequence (beam_state.py:76-98).                        */
int be_beam_add_root(be_trie* t, const int32_t* tokens, int n, int32_t* leaf_out,
                     int32_t* pages_out);
/* BeamState.add_filtered_results (beam_state.py:101-209): frees dead branches,
 * appends / allocates / forks.  Candidate i's children: child_tokens[child_ptr[i]
 * .. child_ptr[i+1]).  new_leaf/new_child (index of the child, to carry its
 * score) in the reference's new-candidate order; copy_src/dst/len: the
 * copy-on-write tail copies (PageTable.copy_block calls, :190-191) to run with
 * be_fork_tail_copy.  Output arrays need child_ptr[ncand] entries.          */
int be_beam_update(be_trie* t, int ncand, const int32_t* cand_leaf, const int32_t* child_ptr,
                   const int32_t* child_tokens, int32_t* new_leaf, int32_t* new_child,
                   int32_t* n_new, int32_t* copy_src, int32_t* copy_dst, int32_t* copy_len,
                   int32_t* n_copies);
/* Decode inputs per candidate (src/beam_engine/beam.py:168-221): query token,
 * append page, append slot (len(leaf)-1), RoPE position (seq len - 1).      */
int be_beam_step_inputs(be_trie* t, int ncand, const int32_t* cand_leaf, int32_t* query_tok,
                        int32_t* write_page, int32_t* write_pos, int32_t* position);
/* BeamState.get_cascade_input (beam_state.py:211-412).  Returns the level count
 * or -status.  Level l: groups level_group_ptr[l]..[l+1]; its qo/kv indptr at
 * [level_group_ptr[l] + l, level_group_ptr[l+1] + l] (one leading 0 per level);
 * last_page_len at [level_group_ptr[l], level_group_ptr[l+1]); pages
 * kv_indices[level_page_ptr[l] .. level_page_ptr[l+1]).                       */
int be_cascade_build(be_trie* t, int ncand, const int32_t* cand_leaf, int cap_levels,
                     int cap_groups, int cap_pages, int32_t* level_group_ptr,
                     int32_t* level_page_ptr, int32_t* qo_indptr, int32_t* kv_indptr,
                     int32_t* kv_indices, int32_t* last_page_len);
/* BeamState._build_kv_tree_structure + _build_req_to_token
 * (beam_state.py:414-564): BFS nodes, request lists, req_to_token slot table
 * [ncand][max_len].  per_node bit 0 stores each node's own length as seqlen
 * (the reference stores the cumulative length); bit 1 makes one tree node of
 * every chain of trie nodes with a single live child (own lengths implied), a
 * layout of this library's tree plans.  req_to_token == NULL: sizes only.   */
int be_tree_build(be_trie* t, int ncand, const int32_t* cand_leaf, int per_node, int page_size,
                  int cap_nodes, int32_t* num_nodes, int32_t* node_parent, int32_t* node_seqlen,
                  int32_t* node_children, int32_t* req_ptr, int32_t* req_list,
                  int64_t cap_req_list, int32_t* max_len, int32_t* req_to_token,
                  int64_t cap_req_to_token);
/* prepare_fasttree_metadata_for_paged_cache
 * (src/beam_engine/attention/fasttree/preparation.py:11-225): cost model,
 * vnodes, req->vnode lists, two-phase order.  counts = {vnodes, entries,
 * phase-0 vnodes, phase-1 vnodes}.                                           */
int be_fasttree_prepare(int num_nodes, const int32_t* node_parent, const int32_t* node_seqlen,
                        const int32_t* node_children, const int32_t* req_ptr,
                        const int32_t* req_list, int64_t req_to_token_stride, int batch_size,
                        int num_qo_heads, int num_kv_heads, int cap_vnodes, int cap_entries,
                        int32_t* q_entries, int32_t* q_offs, int32_t* q_lens, int32_t* kv_offs,
                        int32_t* kv_lens, int32_t* r2v_entries, int32_t* r2v_offs,
                        int32_t* r2v_lens, int32_t* counts);
/* VanillaBeamSearchStrategy.select_candidates (src/beam_engine/beam_strategy.py:433-488).
 * tokens/logps: [n][k] children in top-k order.  Outputs child_ptr [n+1],
 * child_tokens / child_scores [<= beam_size].                                */
int be_vanilla_select(int n, int k, const double* parent_scores, const int32_t* tokens,
                      const double* logps, int beam_size, int32_t* child_ptr,
                      int32_t* child_tokens, double* child_scores);

/* Vanilla selection over several prompts at once (each prompt's candidates
 * seg_ptr[s]..seg_ptr[s+1] keep their own beam_size), the batched form of
 * VanillaBeamSearchStrategy.select_candidates (src/beam_engine/beam_strategy.py:433-488)
 * that the reference calls once per generate().                              */
int be_vanilla_select_segments(int nseg, const int32_t* seg_ptr, int k,
                               const double* parent_scores, const int32_t* tokens,
                               const double* logps, int beam_size, int32_t* child_ptr,
                               int32_t* child_tokens, double* child_scores,
                               int32_t* new_seg_ptr);
/* VanillaBeamSearchStrategy.select_candidates (src/beam_engine/beam_strategy.py:433-488)
 * for every prompt in one launch, on the device: candidates seg_ptr[s] ..
 * seg_ptr[s+1] of prompt s offer their top-k children (logps / tokens
 * [ncand][k], each row sorted as be_logsoftmax_topk writes it) with
 * accumulated score parent_scores[c] + logps[c][j] in double; the prompt keeps
 * the beam_size best of a stable descending sort (ties: earlier candidate,
 * then earlier top-k position).  Out, for slot r < beam_size of prompt s at
 * s * beam_size + r, in rank order: sel_parent (candidate index; -1 past the
 * prompt's entry count), sel_token, sel_score.  All pointers are device
 * memory; every prompt has at most max_seg_cands candidates and
 * max_seg_cands * k <= 8192.                                                  */
int be_vanilla_select_device(int nseg, const int32_t* seg_ptr, int k, const double* parent_scores,
                             const float* logps, const int64_t* tokens, int beam_size,
                             int max_seg_cands, int32_t* sel_parent, int32_t* sel_token,
                             double* sel_score, void* stream);
/* The trie update (be_beam_update, beam_state.py:101-209) from selections in
 * the form be_vanilla_select_device writes (host copies): children per old
 * candidate in rank order, prompts in order.  Same outputs as
 * be_beam_select_update.                                                      */
int be_beam_update_selected(be_trie* t, int nseg, const int32_t* seg_ptr, const int32_t* cand_leaf,
                            const int32_t* sel_parent, const int32_t* sel_token,
                            const double* sel_score, int beam_size, int32_t* new_leaf,
                            double* new_score, int32_t* n_new, int32_t* new_seg_ptr,
                            int32_t* copy_src, int32_t* copy_dst, int32_t* copy_len,
                            int32_t* n_copies, int32_t* child_ptr);
/* DiverseBeamSearchStrategy.select_candidates (src/beam_engine/beam_strategy.py:173-317)
 * for several prompts at once (candidates seg_ptr[s]..seg_ptr[s+1] form prompt s).
 * tokens/logps [ncand][k] in top-k order; seq_ptr [ncand + 1] / seq_tokens are the
 * parents' token sequences (be_leaf_sequences; seq_tokens may be NULL for hamming).
 * diversity_type 0 = "hamming", 1 = "cumulative" (any other reference string).
 * Outputs child_ptr [ncand + 1], child_tokens / child_scores [<= nseg * beam_size]
 * (children per parent in pick order), new_seg_ptr [nseg + 1].              */
int be_diverse_select(int nseg, const int32_t* seg_ptr, int k, const double* parent_scores,
                      const int32_t* tokens, const double* logps, const int32_t* seq_ptr,
                      const int32_t* seq_tokens, int beam_size, int num_groups,
                      double diversity_penalty, int diversity_type, double length_penalty,
                      int32_t* child_ptr, int32_t* child_tokens, double* child_scores,
                      int32_t* new_seg_ptr);
/* be_diverse_select on the device for the hamming penalty (diversity_type 0;
 * DiverseBeamSearchStrategy.select_candidates, src/beam_engine/beam_strategy.py:
 * 173-317 with :105-125): the same arguments and outputs, all pointers device
 * memory, one CTA per prompt.  seq_ptr [ncand + 1] only gives the parents'
 * lengths for the length penalty (no token sequences are read).  Limits:
 * max_seg_cands (the largest prompt's candidate count) * k <= 8192 and
 * num_groups * max(1, beam_size / num_groups) <= 1024; diversity_type 1
 * returns BE_ENOTSUP.  A length_penalty other than 0 or 1 goes through the
 * device pow(), whose last bit may differ from the host's.                   */
int be_diverse_select_device(int nseg, const int32_t* seg_ptr, int k, const double* parent_scores,
                             const int32_t* tokens, const double* logps, const int32_t* seq_ptr,
                             int beam_size, int num_groups, double diversity_penalty,
                             int diversity_type, double length_penalty, int max_seg_cands,
                             int32_t* child_ptr, int32_t* child_tokens, double* child_scores,
                             int32_t* new_seg_ptr, void* stream);

/* ---- Tensor-parallel all-reduce over peer memory (one process per GPU) ----
 * Replaces the NCCL all-reduce after the row-parallel projections
 * (o_proj, down_proj) plus the residual add + RMSNorm that follow it
 * (modeling_llama.py:68-173 decoder layer under tensor parallelism).  Each rank
 * owns `num_slots` data slots in one allocation that the other ranks map
 * through CUDA IPC; the GEMM writes its partial into this rank's slot, then
 * be_comm_allreduce_rmsnorm sums every rank's slot (plain peer loads, no
 * multicast) and applies the residual add and the norm.  Consecutive calls
 * must alternate between two slots.  A rank that stops answering makes the
 * others' barrier time out after 2 s (BE_EDEVICE_TIMEOUT in be_device_status);
 * a CTA whose wait ran out returns without writing its rows, so residual / out
 * of that call are undefined (BeamSearchGenerator raises when the status is
 * set at the end of a tensor-parallel generation).  From 4 ranks on the call
 * runs in a two-shot form (each row reduced by one owner rank, then copied by
 * the others; same results); BE_COMM_TWO_SHOT_WORLD sets the rank count
 * (0: never).                                                                */
typedef struct be_comm be_comm;
#define BE_IPC_HANDLE_BYTES 64
/* Allocate this rank's flags + slots; writes its IPC handle (BE_IPC_HANDLE_BYTES)
 * to handle_out.  max_ctas bounds the CTAs of one call (rows beyond it are
 * strided).  world <= 8.                                                     */
int be_comm_create(int world, int rank, int64_t slot_bytes, int num_slots, int max_ctas,
                   void* handle_out, be_comm** out);
/* Map the other ranks' allocations: handles = world x BE_IPC_HANDLE_BYTES in rank
 * order.  Every rank must have finished be_comm_open before any rank's first
 * be_comm_allreduce_rmsnorm (a host barrier).                                */
int be_comm_open(be_comm* comm, const void* handles);
/* Device address of this rank's slot (where the GEMM writes its partial).    */
void* be_comm_slot(be_comm* comm, int slot);
/* Device address of this rank's incoming flag array: uint32 [max_ctas][8],
 * entry [cta][r] = the call count rank r last signalled for that CTA.  A
 * handle equal to this rank's own (be_comm_open) maps this rank's buffer in
 * that rank's place (loopback, for tests on one GPU).                        */
void* be_comm_flags(be_comm* comm);
/* Unmap the other ranks' allocations (after the last call on every rank).    */
int be_comm_close_peers(be_comm* comm);
/* Free this rank's allocation -- after every other rank closed its mapping of
 * it (a host barrier after be_comm_close_peers on all ranks).                */
int be_comm_destroy(be_comm* comm);
/* sum = sum over ranks of slot[rows][hidden] (fp32, rank order: identical bits
 * on every rank).  residual != NULL: residual += round(sum), out = norm_w *
 * rmsnorm(residual) (be_add_rmsnorm's arithmetic); residual == NULL: out = sum. */
int be_comm_allreduce_rmsnorm(be_comm* comm, int slot, void* residual, const void* norm_w,
                              void* out, int rows, int hidden, float eps, int dtype,
                              void* stream);

/* Vocabulary-parallel scoring over the same peer buffer, replacing the two
 * all-reduces and two all-gathers of the distributed log-softmax / top-k
 * (beam.py:266-317 scoring, with the vocabulary sharded over the ranks).
 * Each rank's be_logsoftmax_topk (full_vocab = 0) writes into this rank's slot
 * at the byte offsets be_comm_topk_layout gives (offsets[0..3]: int64 global
 * ids [rows][k], float values [rows][k], float row max [rows], float row sum of
 * exponentials [rows]); be_comm_topk_merge then writes, on every rank, the
 * global top k as log-probabilities (value desc, id asc) with their ids.
 * k <= 64.  The slot must not be the one the last all-reduce before it used,
 * and the next call that writes this slot must come after another call of
 * this communicator (a slot of its own is simplest).                         */
int be_comm_topk_layout(int rows, int k, int64_t* offsets);
int be_comm_topk_merge(be_comm* comm, int slot, int rows, int k, float* out_val,
                       int64_t* out_idx, void* stream);

/* One host call per decode step after the device's top-k: vanilla selection
 * of every prompt (be_vanilla_select_segments, beam_strategy.py:433-488) then
 * the trie update (be_beam_update, beam_state.py:101-209).  new_leaf /
 * new_score / copy_* need nseg * beam_size entries, new_seg_ptr nseg + 1;
 * child_ptr (may be NULL): the selected children per old candidate as CSR.  */
int be_beam_select_update(be_trie* t, int nseg, const int32_t* seg_ptr, int k,
                          const int32_t* cand_leaf, const double* parent_scores,
                          const int32_t* tokens, const double* logps, int beam_size,
                          int32_t* new_leaf, double* new_score, int32_t* n_new,
                          int32_t* new_seg_ptr, int32_t* copy_src, int32_t* copy_dst,
                          int32_t* copy_len, int32_t* n_copies, int32_t* child_ptr);
/* 1 when some query of a cascade plan attends one page at two levels (the
 * reference's uneven-tree quirk, beam_state.py:299-302), else 0; the picker
 * then takes the tree plan (each page once).  Same level arrays as
 * be_cascade_plan; -BE_EINVAL on bad arguments.                              */
int be_cascade_pages_twice(int num_levels, const int32_t* const* qo_indptr,
                           const int32_t* const* kv_indptr, const int32_t* const* kv_indices,
                           const int32_t* num_groups, int num_queries);

/* One call for a cascade decode step's host inputs (beam.py:168-221 decode
 * inputs + BeamState.get_cascade_input beam_state.py:211-412 + the attention
 * plan): out[0..n) query tokens, [n..2n) RoPE positions, [2n..3n) append
 * pages, [3n..4n) append slots, plan (with header) from out[plan_offset].    */
int be_beam_decode_inputs(be_trie* t, int ncand, const int32_t* cand_leaf, int num_qo_heads,
                          int num_kv_heads, int num_sms, int32_t* out, int64_t cap,
                          int32_t plan_offset, be_attn_plan_info* info);

/* be_beam_decode_inputs with a tile plan (be_tile_plan) from out[plan_offset].
 * BE_ENOTSUP when the step's cascade is not a decode shape.                 */
int be_beam_decode_tiles(be_trie* t, int ncand, const int32_t* cand_leaf, int num_qo_heads,
                         int num_kv_heads, int tile_rows, int target_pieces, int cluster,
                         int32_t* out, int64_t cap, int32_t plan_offset,
                         be_tile_plan_info* info);

#ifdef __cplusplus
}
#endif
#endif /* BEAM_B200_H */
