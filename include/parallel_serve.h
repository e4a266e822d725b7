/*
 * parallel_serve.h — C ABI of the B200 (sm_100a) fused two-model decode path.
 *
 * Two same-architecture models are co-located on one GPU. Their weights are
 * stacked as W[2, K, N] (row-major, N contiguous). Every decode token carries a
 * model id (0 or 1). All entry points take plain device pointers and sizes,
 * launch asynchronously on the given CUDA stream and return a PS_* code for
 * argument errors found on the host. Errors found on the device (a wait that
 * ran out, a model id that is not 0/1, an index out of range) are OR-ed into
 * the caller's device status word (`int32_t* status`, may be NULL) as
 * PS_ERR_* bits; read it after a synchronize.
 *
 * Token order: kernels that take `counts` work on tokens in *routed order*:
 * the counts[0] model-0 tokens first, then the counts[1] model-1 tokens, each
 * group in original (stable) order. ps_route_partition produces the
 * permutation; ps_gather_rows applies it; the GEMM epilogue can scatter back.
 *
 * Element types: `dtype` is PS_DTYPE_F16 or PS_DTYPE_BF16 for every 16-bit
 * activation / weight buffer of a call; accumulation is always fp32.
 *
 * Reference interfaces replaced (paths within the reference project):
 *   routed_gemm(x, W_stacked, split_point)      kernel/src/routed_gemm.py:152-197
 *   routed_linear_n2(x, W_stacked, split_point) experiments/routed_linear_n2.py:118-153
 *   TwoModelBlockRouted._rms_norm_per_model     kernel/src/two_model_block_routed.py:89-98
 *   TwoModelBlockRouted._sdpa_per_model         kernel/src/two_model_block_routed.py:100-120
 *   TransformerBlock.forward (norm/attn/silu)   experiments/two_model_block.py:54-74
 *   DeltaZip base+delta linear (Marlin-24 acc)  docs/deltazip_progress_2026-04-17.md:154-162
 */
#ifndef PARALLEL_SERVE_H_
#define PARALLEL_SERVE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- host return codes ---------------------------------------------------- */
#define PS_OK 0
#define PS_ERR_INVALID_ARGUMENT 1 /* shape / pointer / alignment check failed */
#define PS_ERR_WORKSPACE 2        /* workspace missing or too small            */
#define PS_ERR_CUDA 3             /* a CUDA runtime / driver call failed        */
#define PS_ERR_UNSUPPORTED 4      /* device is not sm_100 or size beyond limit  */
#define PS_ERR_SCRATCH_LIMIT 5    /* problem needs more than the static scratch */

/* ---- device status bits (OR-ed into *status) ------------------------------ */
#define PS_ERR_TIMEOUT 0x1      /* a bounded wait inside a kernel ran out      */
#define PS_ERR_BAD_MODEL_ID 0x2 /* a model id other than 0 or 1 was seen       */
#define PS_ERR_BAD_INDEX 0x4    /* a token / slot / position index out of range */

#define PS_DTYPE_F16 0
#define PS_DTYPE_BF16 1

/* Epilogue modes of ps_routed_gemm. */
#define PS_EPI_STORE 0  /* y = acc (+ residual)                                  */
#define PS_EPI_SWIGLU 1 /* W columns are [gate | up] (N = 2*FF): y[:, f] =
                           silu(acc_gate[f]) * acc_up[f], y has FF columns      */
#define PS_EPI_QKV_ROPE 2 /* ps_routed_gemm_ex only: W columns are [q | k | v],
                             128 per head; q (rotated) -> y, k (rotated) and v
                             appended to the token's model KV pools          */

typedef void* ps_stream_t; /* a cudaStream_t */

/* Human-readable name of a PS_* return code. */
const char* ps_error_string(int code);

/* Library version string and the sm_100a build marker. */
const char* ps_version(void);

/* Streaming multiprocessor count of `device` (cached after the first call). */
int ps_device_sm_count(int device);

/* ------------------------------------------------------------------------- *
 * Route bookkeeping (an addition of this library; the reference only has a
 * host int split_point, kernel/src/routed_gemm.py:157).
 *
 * Stable partition of `model_id[M]` (values 0/1): perm[j] = original index of
 * the j-th token in routed order; counts[0..1] = tokens per model. Bit-exact
 * with a stable argsort of model_id. Ids outside {0,1} set PS_ERR_BAD_MODEL_ID.
 * ------------------------------------------------------------------------- */
int ps_route_partition(const int32_t* model_id, int M, int32_t* perm, int32_t* counts,
                       int32_t* status, ps_stream_t stream);

/* dst[j, :] = src[perm[j], :] for j < M; rows of row_bytes bytes (multiple of 16). */
int ps_gather_rows(const void* src, const int32_t* perm, void* dst, int M, int row_bytes,
                   int32_t* status, ps_stream_t stream);

/* dst[perm[j], :] = src[j, :] for j < M. */
int ps_scatter_rows(const void* src, const int32_t* perm, void* dst, int M, int row_bytes,
                    int32_t* status, ps_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Routed GEMM — replaces routed_gemm / routed_linear_n2
 * (kernel/src/routed_gemm.py:152-197, experiments/routed_linear_n2.py:118-153).
 *
 *   rows [0, c0) of x use W[0], rows [c0, c0+c1) use W[1], where
 *   (c0, c1) = counts[0..1] read on the device when `counts` != NULL (one
 *   CUDA graph then serves every split), else (split_point, M - split_point).
 *
 * x [M, K] row-major; W [2, K, N] row-major; y [M, N] (PS_EPI_STORE) or
 * [M, N/2] (PS_EPI_SWIGLU), row-major. Output row j is written to
 * y[scatter_rows ? scatter_rows[j] : j] (a row outside [0, M) is skipped and
 * sets PS_ERR_BAD_INDEX). `residual` (nullable, same shape and
 * row mapping as y, may alias y) is added before the store.
 * With counts == NULL and split_point == M only W[0] is read, so W may be a
 * single [K, N] matrix (the serial per-model path).
 * K % 8 == 0, N % 8 == 0 (N/2 % 8 == 0 for SWIGLU), 16-byte aligned pointers.
 * `workspace` (size from ps_routed_gemm_workspace_bytes) holds a fixed
 * 256 KiB region of per-tile arrival counters followed by stream-K partial
 * tiles. Zero-fill it once before its first use: kernels leave the counter
 * region zeroed, so the same buffer serves later calls of any shape. It must
 * not be shared by kernels that run concurrently.
 * ------------------------------------------------------------------------- */
size_t ps_routed_gemm_workspace_bytes(int M, int N, int epilogue, int device);

int ps_routed_gemm(const void* x, const void* W, void* y, int M, int K, int N,
                   int split_point, const int32_t* counts, const int32_t* scatter_rows,
                   const void* residual, int epilogue, int dtype, void* workspace,
                   size_t workspace_bytes, int32_t* status, ps_stream_t stream);

/* Same computation as ps_routed_gemm, for callers that cannot provide or
 * allocate device memory (a runtime whose pool owns all device memory, a
 * plugin host that forbids allocation during execution, a loop that cannot
 * afford the synchronisation cudaMalloc may cause). It has no counterpart in
 * the reference. Scratch comes from a 16 MiB array inside this library that
 * every GPU loading the library holds until exit; nothing is allocated. The
 * first call on a device resolves that array's address (make it before any
 * stream capture; host threads making first calls at once are serialised by
 * the library). Limit: 16384 output tiles (128 weight columns x 128
 * tokens of one model each) per call, else PS_ERR_SCRATCH_LIMIT; with more
 * than 96 rows (M) fewer CTAs run. All calls share the array: calls that
 * overlap on the GPU race. */
int ps_routed_gemm_noalloc(const void* x, const void* W, void* y, int M, int K, int N,
                           int split_point, const int32_t* counts, const int32_t* scatter_rows,
                           const void* residual, int epilogue, int dtype, int32_t* status,
                           ps_stream_t stream);

/* Schedule introspection (host only, no CUDA call): the routed GEMM kernel's
 * own schedule functions, run on the host for a launch with c0 / c1 tokens of
 * model 0 / 1, K, N, the epilogue mode and `grid` CTAs, so that tests and
 * tuning can check what each CTA does.
 *   ps_routed_gemm_schedule: info[10] = {T0, T1 (token tiles per model),
 *     weight tiles per token tile, tiles, k-blocks per tile, iterations,
 *     stream-K range length, data-parallel rounds, first stream-K iteration,
 *     grid}.
 *   ps_routed_gemm_cta_work: CTA `cta`'s pieces in execution order, 6 ints
 *     each {tile, first k-block, end k-block, partial slot (-1: whole tile,
 *     0 / 1: the slot its fp32 partial goes to), first and last CTA
 *     contributing to the tile (-1 for whole tiles)}; writes at most `cap`
 *     pieces, returns the number of pieces (or a negative error code).
 *   ps_routed_gemm_tile: tile t's {model, first row, tokens, first weight
 *     column, second 64-column half's first column, first output column}. */
int ps_routed_gemm_schedule(int c0, int c1, int K, int N, int epilogue, int grid, int32_t* info);
int ps_routed_gemm_cta_work(int c0, int c1, int K, int N, int epilogue, int grid, int cta,
                            int32_t* pieces, int cap);
int ps_routed_gemm_tile(int c0, int c1, int K, int N, int epilogue, int grid, int t,
                        int32_t* out);

/* ------------------------------------------------------------------------- *
 * Routed GEMM with a fused decode-layer epilogue. Replaces, in one launch,
 * the sequences the reference runs as separate ops around each projection of
 * kernel/src/two_model_block_routed.py:120-160 and
 * experiments/two_model_block.py:55-75:
 *   RMSNorm -> projection          (in_sumsq, norm weight folded into W)
 *   projection -> RoPE -> KV write (PS_EPI_QKV_ROPE)
 *   projection + residual -> the next RMSNorm's sum of squares (out_sumsq)
 *
 * Folded RMSNorm: rms_norm(x) @ W == diag(rstd) (x @ (diag(w) W)) with
 * rstd[j] = 1/sqrt(sum(x[j]^2)/norm_dim + eps). The caller scales the rows of
 * W by the norm weight w once at load; the kernel multiplies accumulator
 * column j by rstd[j], the squares coming as in_parts partial sums per row,
 * in_sumsq[j * in_parts + p], added in order p = 0, 1, ... (reproducible).
 * out_sumsq (PS_EPI_STORE only) receives such partials for the stored
 * (rounded) output: out_sumsq[row * ceil(N/128) + t] = sum of squares of
 * output features [128t, 128t + 128) of that row, written once each (no
 * atomics, no zeroing; feed it to the next launch with in_parts = ceil(N/128)).
 *
 * PS_EPI_QKV_ROPE: N == 3 * n_heads * 128 and y is [M, n_heads * 128] (q).
 * For routed row j of model m: position p = pos[j], slot s = j - (m ? c0 : 0);
 * q, k are rotated with rope_cos/sin[p, 0..63] (rotate-half convention) when
 * apply_rope, k -> k_pool_m[s, h, p, :], v -> v_pool_m[s, h, p, :] (pools
 * [slots, n_heads, L_cap, 128]). Out-of-range s or p set PS_ERR_BAD_INDEX.
 * Other arguments as in ps_routed_gemm; the workspace size is
 * ps_routed_gemm_workspace_bytes(M, N, mode == PS_EPI_SWIGLU, device).
 * ------------------------------------------------------------------------- */
typedef struct ps_gemm_epilogue {
  int mode;                    /* PS_EPI_STORE / PS_EPI_SWIGLU / PS_EPI_QKV_ROPE */
  const int32_t* scatter_rows; /* STORE / SWIGLU, nullable                         */
  const void* residual;        /* STORE, nullable, may alias y                     */
  const float* in_sumsq;       /* nullable: folded RMSNorm of the rows of x        */
  int in_parts;                /* partial sums per row in in_sumsq                 */
  int norm_dim;                /* elements per row of x behind in_sumsq            */
  float eps;
  float* out_sumsq; /* STORE, nullable: [rows of y][ceil(N/128)] fp32 partials    */
  void* k_pool0; /* QKV_ROPE: model 0 / model 1 KV pools                         */
  void* v_pool0;
  void* k_pool1;
  void* v_pool1;
  const int32_t* pos;     /* QKV_ROPE: [M] position of routed row j               */
  const float* rope_cos;  /* QKV_ROPE: [L_cap (paged: max_pages*page_size), 64]   */
  const float* rope_sin;
  int n_heads, L_cap, slots0, slots1, apply_rope;
  /* QKV_ROPE into paged pools (nullable): pools are [pages, n_heads,
   * page_size, 128], k/v of routed row j at position p go to page
   * block_table[j*max_pages + p/page_size], row p % page_size; slots0 /
   * slots1 are then the pools' page counts and L_cap is ignored. */
  const int32_t* block_table;
  int max_pages, page_size;
  /* QKV_ROPE (nullable): kv_rows[j] = the KV home of routed row j — its slot in
   * model m(j)'s contiguous pool, or its block-table row for paged pools —
   * when several rows (prompt tokens of one sequence in a prefill) share one
   * sequence. NULL: slot j - (m ? c0 : 0), block-table row j. Block-table
   * rows must be below table_rows (else PS_ERR_BAD_INDEX, no write). */
  const int32_t* kv_rows;
  int table_rows;
  /* Upper bound on the rows of either model in this call (0 = M): a bound
   * below M narrows each pipeline stage's x tile, so more weight stages fit
   * (decode: the larger model's batch). Rows beyond it stay correct (more
   * token tiles), only slower. The projection chain requires it to hold. */
  int max_model_rows;
  /* Nullable: the same weights packed by ps_pack_weights for this epilogue
   * mode; the kernel then streams each stage's weights as one contiguous
   * 32 KB block (W may be NULL). */
  const void* w_packed;
  /* CTAs of the launch: 0 = one per SM; > 0 = at most this many; -1 = chosen
   * for the shape: small projections (tensor-parallel shards) lose less to
   * split-tile fix-up with whole tiles per CTA (short K) or tiles split into
   * equal aligned pieces, large ones keep every SM. */
  int max_ctas;
} ps_gemm_epilogue_t;

int ps_routed_gemm_ex(const void* x, const void* W, void* y, int M, int K, int N,
                      int split_point, const int32_t* counts, const ps_gemm_epilogue_t* epi,
                      int dtype, void* workspace, size_t workspace_bytes, int32_t* status,
                      ps_stream_t stream);

/* Packed weights for the routed GEMM (an HBM layout of this library; the
 * reference keeps W [2, K, N] and so does every entry point that takes W).
 * Each (model, weight tile of 128 columns — SwiGLU: 64 gate + their 64 up
 * columns —, 128-k block) becomes one contiguous 32 KB block holding the
 * pipeline stage's shared-memory image (128-byte swizzled, zero past K and
 * N), so a stage is one sequential bulk read. nmat = 2 for stacked weights.
 * The packing depends on the epilogue mode (SwiGLU pairs columns). */
size_t ps_packed_weights_bytes(int nmat, int K, int N, int epilogue);

int ps_pack_weights(const void* W, int nmat, int K, int N, int epilogue, void* out,
                    size_t out_bytes, ps_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Projection chain: several routed GEMMs of one decode layer (and, under
 * tensor parallelism, the all-reduces of the row-split ones) in ONE
 * persistent launch. Replaces the reference's sequence of per-projection
 * routed GEMM calls between two attentions, kernel/src/two_model_block_routed.py:
 * 138-152 (O + residual, RMSNorm, gate_up, SwiGLU, down + residual), plus the
 * next layer's QKV (or the LM head); the reference launches ~15 kernels per
 * layer for this and has no multi-GPU path.
 *
 * A job is either a routed GEMM (x @ W with the fused epilogue of
 * ps_routed_gemm_ex) or an all-reduce of a row-split GEMM's partial that job
 * `src` wrote into this rank's symmetric slot `slot`:
 *   out = residual + sum over ranks of the slot  (rows in routed order,
 *   row_elems columns; out_sumsq[row * (row_elems / 64) + u] = sum of squares
 *   of the stored 64-column part u, the next folded RMSNorm's input).
 * Jobs run in order, but without a grid-wide wait between them: every
 * 64-column part of a job's output, once final, is published with a counter,
 * and a later job waits only for the parts it reads:
 *   x_from    job whose output is this GEMM's x: each 128-k block of x waits
 *             for its two parts (weights keep streaming meanwhile);
 *   norm_from job that wrote epi.in_sumsq: the epilogue waits for all parts;
 *   res_from  job that wrote epi.residual (GEMM) / residual (all-reduce): the
 *             tile's parts are awaited before they are read;
 * -1 means the data was complete before the launch. Every job routes by the
 * device `counts` (both models <= 128 rows: decode batches). Results are
 * identical to the same GEMMs launched one by one (same stream-K cut, same
 * summation order); the chain's all-reduce sums ranks in order 0..world-1.
 * Waits are bounded (PS_ERR_TIMEOUT). At most 6 jobs; outputs of at most
 * 32768 columns. The workspace (ps_routed_chain_workspace_bytes, zero-filled
 * once) keeps a launch epoch and must not be shared by concurrent calls.
 * ------------------------------------------------------------------------- */
#define PS_JOB_GEMM 0
#define PS_JOB_ALLREDUCE 1
typedef struct ps_chain_job_t {
  int kind;
  /* PS_JOB_GEMM: y[M, N'] = x[M, K] @ W[2, K, N] routed, epilogue `epi` */
  const void* x;
  const void* W;
  void* y;
  int K, N;
  ps_gemm_epilogue_t epi;
  int x_from, norm_from, res_from;
  /* PS_JOB_ALLREDUCE */
  int src, slot;
  void* out;
  const void* residual;
  float* out_sumsq;
  int row_elems;
} ps_chain_job_t;

size_t ps_routed_chain_workspace_bytes(int M, int n_jobs, int device);

/* peer_bases / rank / world / slot_bytes as for ps_allreduce_sum (world = 1
 * and peer_bases = {this rank's region} when the chain has no all-reduce;
 * peer_bases may be NULL then). */
int ps_routed_chain(const ps_chain_job_t* jobs, int n_jobs, int M, const int32_t* counts,
                    void* const* peer_bases, int rank, int world, size_t slot_bytes, int dtype,
                    void* workspace, size_t workspace_bytes, int32_t* status,
                    ps_stream_t stream);


/* ------------------------------------------------------------------------- *
 * Per-model RMSNorm — replaces _rms_norm_per_model
 * (kernel/src/two_model_block_routed.py:89-98) and the F.rms_norm calls of
 * experiments/two_model_block.py:56,69.
 *   y[j] = x[j] / sqrt(mean(x[j]^2) + eps) * w[m(j)],  m(j) = j >= c0
 * w is [2, H]. counts / split_point as in ps_routed_gemm.
 * ------------------------------------------------------------------------- */
int ps_rmsnorm_routed(const void* x, const void* w, void* y, int M, int H, int split_point,
                      const int32_t* counts, float eps, int dtype, int32_t* status,
                      ps_stream_t stream);

/* SwiGLU: out[j, f] = silu(gu[j, f]) * gu[j, FF + f]  (experiments/two_model_block.py:71-72). */
int ps_swiglu(const void* gu, void* out, int M, int FF, int dtype, ps_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Decode KV cache. Each model owns a K pool and a V pool laid out
 * [slots, n_heads, L_cap, head_dim] (head_dim = 128), so one (slot, head)
 * stream is contiguous. Token j (routed order) belongs to model m(j) and uses
 * pool slot `slot[j]` (or j - offset(m(j)) when slot == NULL); `pos[j]` is the
 * position of its new token (= number of cached tokens before this step).
 * ------------------------------------------------------------------------- */

/* RoPE (rotate-half, cos/sin table [L_cap, head_dim/2] fp32) on q and the new
 * k from qkv [M, 3*n_heads*128]; writes q_out [M, n_heads*128] and appends
 * k, v at position pos[j] of the token's pools. (An addition of this library:
 * the reference has no RoPE or KV cache, experiments/real_weights_full_stack.py:11.) */
int ps_rope_kv_append(const void* qkv, void* q_out, void* k_pool0, void* v_pool0,
                      void* k_pool1, void* v_pool1, const float* rope_cos,
                      const float* rope_sin, const int32_t* pos, const int32_t* slot,
                      const int32_t* counts, int split_point, int M, int n_heads, int L_cap,
                      int slots0, int slots1, int apply_rope, int dtype, int32_t* status,
                      ps_stream_t stream);

/* Fused two-model decode attention (flash-decoding): for token j and head h,
 * out[j, h] = softmax(q[j,h] . K[0..pos[j]] * scale) V[0..pos[j]] over the
 * token's own pool (model-id dispatch), split over the sequence in chunks of
 * `chunk` positions (0 = choose). Replaces F.scaled_dot_product_attention in
 * TwoModelBlockRouted._sdpa_per_model (kernel/src/two_model_block_routed.py:100-120)
 * for decode. max_len bounds pos[j]+1 (sizes the grid). */
size_t ps_decode_attention_workspace_bytes(int M, int n_heads, int max_len, int chunk);

int ps_decode_attention(const void* q, const void* k_pool0, const void* v_pool0,
                        const void* k_pool1, const void* v_pool1, void* out,
                        const int32_t* pos, const int32_t* slot, const int32_t* counts,
                        int split_point, int M, int n_heads, int L_cap, int slots0,
                        int slots1, int max_len, int chunk, float scale, int dtype,
                        void* workspace, size_t workspace_bytes, int32_t* status,
                        ps_stream_t stream);

/* Paged variant (the production decode layout; the reference keeps one
 * contiguous cache per sequence, kernel/FRIDAY_REPORT.md:131). Each model's K
 * and V live in page pools [pages_m, n_heads, page_size, 128]; block_table
 * [M, max_pages] int32 maps routed row j's positions [i*page_size,
 * (i+1)*page_size) to page block_table[j*max_pages + i] of model m(j)'s pool.
 * page_size is a power of two in [8, 4096]; pos[j] < max_pages*page_size.
 * seq_rows (nullable) maps row j to its block-table row (prompt tokens of one
 * sequence in a prefill share a row; NULL: row j); block_table has table_rows
 * rows (a row index outside them sets PS_ERR_BAD_INDEX). A page id outside
 * [0, pages_m) sets PS_ERR_BAD_INDEX and that (token, head, chunk) is skipped. Same math and chunking as ps_decode_attention, so the
 * output is bit-identical to the contiguous call on the same K/V. */
size_t ps_paged_decode_attention_workspace_bytes(int M, int n_heads, int max_len, int chunk,
                                                 int page_size);

int ps_paged_decode_attention(const void* q, const void* k_pages0, const void* v_pages0,
                              const void* k_pages1, const void* v_pages1, void* out,
                              const int32_t* pos, const int32_t* block_table, int table_rows,
                              const int32_t* seq_rows, int max_pages,
                              int page_size, const int32_t* counts, int split_point, int M,
                              int n_heads, int pages0, int pages1, int max_len, int chunk,
                              float scale, int dtype, void* workspace, size_t workspace_bytes,
                              int32_t* status, ps_stream_t stream);

/* Causal prefill attention on the tensor cores (no counterpart in the
 * reference, which measures decode only; its prefill plan is a varlen causal
 * attention, docs/routing_kernel_design.md:229-232). The prompt tokens'
 * k / v are already in the contiguous KV pools (QKV epilogue of the same
 * routed chunk). blocks: int32 [nblocks][5] = {row0, nq, p0, model, slot}:
 * q rows row0 .. row0+nq-1 (nq <= 128) are prompt tokens at positions
 * p0 .. p0+nq-1 of the sequence in `slot` of `model`'s pool; each attends to
 * its pool positions [0, its own position]. q, out: [T, n_heads*128]. A block
 * outside its pool or rows sets PS_ERR_BAD_INDEX and is skipped. Paged pools
 * (block_table != NULL, as in ps_paged_decode_attention: pools [pages,
 * n_heads, page_size, 128], slots0 / slots1 = page counts, L_cap =
 * max_pages * page_size): a block's `slot` is its block-table row (< table_rows). */
int ps_prefill_attention(const void* q, const void* k_pool0, const void* v_pool0,
                         const void* k_pool1, const void* v_pool1, void* out,
                         const int32_t* blocks, int nblocks, int T, int n_heads, int L_cap,
                         int slots0, int slots1, const int32_t* block_table, int table_rows,
                         int max_pages, int page_size, float scale, int dtype, int32_t* status,
                         ps_stream_t stream);

/* Segment self-attention with the reference's no-KV semantics
 * (kernel/src/two_model_block_routed.py:100-120, experiments/two_model_block.py:61-65):
 * every token of model m attends (non-causally) to all tokens of model m's
 * segment. qkv [M, 3*n_heads*128] routed order; out [M, n_heads*128]. */
int ps_segment_attention(const void* qkv, void* out, int M, int n_heads, int split_point,
                         const int32_t* counts, float scale, int dtype, int32_t* status,
                         ps_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Route-A DeltaZip linear — replaces the base GEMM + Marlin-24
 * gptq_marlin_24_gemm_acc pair of docs/deltazip_progress_2026-04-17.md:154-162
 * (external vLLM fork, no source in the reference).
 *
 *   y[:c0] = x[:c0] @ W_base,  y[c0:] = x[c0:] @ (W_base + deq(D))
 *
 * W_base [K, N] row-major; deq(D)[k, n] = q[k, n] * scale[k / 128, n] with two
 * kept q in [-7, 7] per group of 4 consecutive k. packed_delta holds, for
 * every 128-column tile t and 64-k block b, 3328 bytes at offset
 * (t * K/64 + b) * 3328: 128 columns x 16 B of kept int4 values (k order,
 * low nibble first), 128 x 8 B of their 2-bit positions in each group of 4,
 * 128 x fp16 scale of the block's 128-group. K % 128 == 0, N % 8 == 0;
 * c0 + c1 <= 112 (or <= 128 tokens of one kind). The W_base tile is read once
 * for both token groups.
 * ------------------------------------------------------------------------- */
size_t ps_deltazip_packed_bytes(int K, int N);

size_t ps_deltazip_workspace_bytes(int M, int N, int device);

int ps_deltazip_linear(const void* x, const void* W_base, const void* packed_delta, void* y,
                       int M, int K, int N, int split_point, const int32_t* counts, int dtype,
                       void* workspace, size_t workspace_bytes, int32_t* status,
                       ps_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Tensor-parallel collective over NVLink peer memory (Megatron-style tensor
 * parallelism: the row-split O / down outputs are summed across ranks; the
 * reference has no multi-GPU code). Each rank allocates one symmetric region with
 * ps_symm_alloc (size ps_symm_region_bytes(slot_bytes)), exchanges the 64-byte
 * IPC handle, and maps the peers' regions with ps_symm_open. A row-split GEMM
 * writes its partial [count] into the local slot `slot` (byte offset
 * ps_symm_slot_offset(slot, slot_bytes) of the region); every rank then calls
 * ps_allreduce_sum with the same arguments except `rank`:
 *   out = residual (nullable) + sum over ranks 0..world-1 of the slot,
 * in fp32, bit-identical on every rank. Consecutive calls must alternate the
 * slot. `epochs` is a zeroed device int32[128] private to the rank. Waits for
 * peers are bounded (1 s; PS_ERR_TIMEOUT in *status).
 * ------------------------------------------------------------------------- */
size_t ps_symm_region_bytes(size_t slot_bytes);

int ps_symm_alloc(size_t bytes, void** ptr, void* ipc_handle);

int ps_symm_open(const void* ipc_handle, void** peer_ptr);

int ps_symm_close(void* peer_ptr);

int ps_symm_free(void* ptr);

/* Optional fused RMSNorm statistics (ps_routed_gemm_ex's in_sumsq with
 * in_parts = row_elems / 256): out_sumsq[row * (row_elems/256) + t] = sum of
 * squares of the stored output elements [256t, 256t + 256) of that row
 * (row_elems % 256 == 0). Pass NULL to skip. */
/* algo: PS_AR_ONE_SHOT reads every rank's whole slot; PS_AR_TWO_SHOT reduces
 * this rank's 1/world share, pushes it into every rank's gather buffer and
 * copies the gathered vector after a second signal / wait round;
 * PS_AR_TWO_SHOT_LL pushes the share as 8-byte {data, epoch} words that the
 * receivers poll, with no second round. The two-shot forms need
 * count % (world * 256) == 0, else one-shot runs; PS_AR_AUTO is one-shot.
 * All sum ranks in order 0..world-1 (bit-identical results). */
#define PS_AR_AUTO 0
#define PS_AR_ONE_SHOT 1
#define PS_AR_TWO_SHOT 2
#define PS_AR_TWO_SHOT_LL 3
int ps_allreduce_sum(void* const* peer_bases, int rank, int world, int slot, size_t slot_bytes,
                     size_t count, void* out, const void* residual, int* epochs, int row_elems,
                     float* out_sumsq, int algo, int dtype, int32_t* status,
                     ps_stream_t stream);

/* Byte offset of data slot `slot` (0 or 1) inside a symmetric region. */
size_t ps_symm_slot_offset(int slot, size_t slot_bytes);

/* Vocab-parallel greedy pick (replaces the reference's single-GPU argmax over
 * full logits; the reference has no tensor parallelism). Every rank holds the
 * logits of its vocabulary shard, logits [M, V_local] (rank r: global indices
 * [r * V_local, (r + 1) * V_local)), rows in routed order. Each row's local
 * (max, index) is exchanged through the symmetric regions (same peer_bases /
 * slot_bytes as ps_allreduce_sum), and every rank writes the same pick, the
 * largest value with the lowest global index on ties:
 *   next_tokens[perm[j]] = pick; tokens_out[perm[j]] = pick (nullable);
 *   seq_len[perm[j]] += 1 (nullable).
 * M <= 4096. `epochs` is a zeroed device int32[M] private to the rank, kept
 * across calls. Waits for peers are bounded (1 s; PS_ERR_TIMEOUT). */
int ps_argmax_tp(const void* logits, const int32_t* perm, int32_t* next_tokens,
                 int32_t* tokens_out, int32_t* seq_len, int M, int V_local,
                 void* const* peer_bases, int rank, int world, size_t slot_bytes, int* epochs,
                 int dtype, int32_t* status, ps_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Decode-step glue.
 * ------------------------------------------------------------------------- */

/* x[j] = emb[m(j)][tokens[perm[j]]] ; emb [2, vocab, H]; x [M, H] routed order.
 * Nullable out_sumsq[j] = sum of squares of x[j] (fp32; one partial per row
 * for the first layer's folded RMSNorm). */
int ps_embed_routed(const void* emb, const int32_t* tokens, const int32_t* perm,
                    const int32_t* counts, void* x, int M, int H, int vocab, float* out_sumsq,
                    int dtype, int32_t* status, ps_stream_t stream);

/* Greedy pick: next[perm ? perm[j] : j] = argmax_v logits[j, v] (first index on
 * ties); if seq_len != NULL, seq_len[perm[j]] += 1. */
int ps_argmax_rows(const void* logits, const int32_t* perm, int32_t* next_tokens,
                   int32_t* seq_len, int M, int V, int dtype, ps_stream_t stream);

/* pos_out[j] = seq_len[perm[j]] (positions of this step's tokens in routed order). */
int ps_positions_routed(const int32_t* seq_len, const int32_t* perm, int32_t* pos_out, int M,
                        ps_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PARALLEL_SERVE_H_ */
