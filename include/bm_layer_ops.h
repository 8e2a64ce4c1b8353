/*
 * bm_layer_ops.h — C ABI of the B200 (sm_100a) fused transformer-layer kernels.
 *
 * The memory-bound per-token ops of a Llama layer, batched over rows (tokens):
 * token-embedding gather, RMSNorm (optionally fused with the residual add),
 * RoPE on Q and the GQA K heads written into a static KV cache, and SwiGLU.
 *
 * Conventions shared by every entry point:
 *   - Plain pointers and sizes only. Every data pointer is a device pointer on
 *     the CUDA device that is current on the calling thread; `stream` is a
 *     cudaStream_t of that device passed as void* (NULL = legacy default stream).
 *   - Launches are asynchronous and stream-ordered; no entry point synchronises,
 *     except bm_status_read, which says so.
 *   - Nothing allocates device memory, except bm_rope_table_create.
 *   - The return value is a bm_status_t. Host-side argument checks happen before
 *     any launch: on failure nothing is launched. No entry point calls exit().
 *   - Data types: BM_F32 (IEEE fp32) or BM_BF16 (bfloat16 storage, 2 bytes).
 *     Arithmetic is fp32 in every kernel; outputs are rounded to nearest-even.
 *   - Rows are dense and row-major unless a stride argument says otherwise.
 *     16-byte aligned pointers with 16-byte multiple row pitches take the
 *     128-bit vector path; anything else runs a scalar path with the same
 *     results.
 *   - Values that only the device can check (token ids, positions and sequence
 *     ids held in device arrays) are checked by the kernels. A bad row is skipped
 *     (its outputs are left unwritten) and a BM_DEVERR_* bit is OR-ed into
 *     *d_status when d_status is not NULL. Read it with bm_status_read.
 *
 * Each entry point cites the reference interface it replaces
 * (NolanKisser/BareMetalInferenceEngine, paths within that project).
 */
#ifndef BM_LAYER_OPS_H
#define BM_LAYER_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BM_ABI_VERSION 1

typedef enum bm_dtype {
  BM_F32 = 0,
  BM_BF16 = 1
} bm_dtype_t;

typedef enum bm_status {
  BM_OK = 0,
  BM_ERR_INVALID_ARGUMENT = 1, /* a size, pointer or dtype fails a host-side check */
  BM_ERR_CUDA = 2,             /* a CUDA runtime call or launch failed */
  BM_ERR_DEVICE = 3            /* bm_status_read found BM_DEVERR_* bits set */
} bm_status_t;

/* Bits a kernel OR-s into *d_status. */
#define BM_DEVERR_BAD_ID 0x1       /* token id outside [0, vocab) */
#define BM_DEVERR_BAD_POSITION 0x2 /* position outside [0, max_seq) or beyond the RoPE table */
#define BM_DEVERR_BAD_SEQUENCE 0x4 /* sequence id outside [0, num_seqs) */
#define BM_DEVERR_TIMEOUT 0x8      /* a tensor-core pipeline wait passed its time limit; outputs incomplete */

/* Human-readable name of a bm_status_t. Never NULL. */
const char* bm_status_string(int status);

/* BM_ABI_VERSION of the loaded library. */
int bm_abi_version(void);

/* Message of the last BM_ERR_* returned on this host thread ("" if none). */
const char* bm_last_error_message(void);

/* Synchronises `stream`, copies *d_status into *flags_out (host) and clears
 * *d_status to 0. Returns BM_ERR_DEVICE when any bit was set, else BM_OK. */
int bm_status_read(int32_t* d_status, int32_t* flags_out, void* stream);

/* ---------------------------------------------------------------------------
 * Embedding gather: out[r, :] = table[ids[r], :]  (bit-exact copy).
 * Replaces the per-token row copy in ExecutionEngine::run_layers
 * (src/execution_engine.cu:98-99) and the host id check of forward()
 * (src/execution_engine.cu:63-65), which becomes BM_DEVERR_BAD_ID.
 * table: [vocab][dim]; out: rows of `dim` elements, `out_row_stride` elements
 * apart (>= dim).
 */
int bm_embed_gather(void* out, const void* table, const int32_t* ids,
                    int64_t rows, int64_t dim, int64_t vocab,
                    int64_t out_row_stride, bm_dtype_t dtype,
                    int32_t* d_status, void* stream);

/* ---------------------------------------------------------------------------
 * RMSNorm over rows: out[r,i] = in[r,i] * rsqrt(mean_i(in[r,:]^2) + eps) * weight[i].
 * Replaces launch_rms_norm (include/kernels.cuh:9, src/kernels.cu:59-78), which
 * normalises one vector per launch. out may equal in (in place).
 * in/out rows are in_stride / out_stride elements apart (>= dim).
 */
int bm_rmsnorm(void* out, const void* in, const void* weight,
               int64_t rows, int64_t dim, float eps,
               int64_t in_stride, int64_t out_stride,
               bm_dtype_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Fused residual add + RMSNorm:
 *   residual[r,:] <- residual[r,:] + delta[r,:]      (fp32 add, stored in dtype)
 *   out[r,:]       = rmsnorm(residual[r,:]) * weight (on the stored values)
 * Replaces the pair launch_add(hidden, hidden, projected) followed by
 * launch_rms_norm(normed, hidden, w) (src/execution_engine.cu:118+121 and
 * :126+:109/:80; include/kernels.cuh:9,32). Rows are dense ([rows][dim]).
 * out must not overlap residual or delta.
 */
int bm_add_rmsnorm(void* residual, const void* delta, const void* weight,
                   void* out, int64_t rows, int64_t dim, float eps,
                   bm_dtype_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Element-wise add: out = a + b over n elements. out may equal a or b.
 * Replaces launch_add (include/kernels.cuh:32, src/kernels.cu:199-207).
 */
int bm_add(void* out, const void* a, const void* b, int64_t n,
           bm_dtype_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * SwiGLU: out = silu(gate) * up = gate / (1 + exp(-gate)) * up over n elements.
 * Replaces launch_swiglu (include/kernels.cuh:29, src/kernels.cu:185-195).
 * out may equal gate or up.
 */
int bm_swiglu(void* out, const void* gate, const void* up, int64_t n,
              bm_dtype_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * One layer step: the five ops above in the order ExecutionEngine::run_layers
 * issues them for a token (src/execution_engine.cu:98-126), for a batch of
 * rows, equivalent to
 *   bm_embed_gather(hidden <- embed[ids])
 *   bm_add_rmsnorm(hidden += attn_out; y_attn = rmsnorm(hidden) * w_attn)
 *   bm_rope_kv_store(q in place; rotated k and v into the caches)
 *   bm_add_rmsnorm(hidden += ffn_out; y_ffn = rmsnorm(hidden) * w_ffn)
 *   bm_swiglu(act = silu(gate) * up)
 * No single reference function: it groups the reference's per-token calls.
 * Every input (the GEMM and attention outputs included) must be ready when it is
 * called; inside one transformer layer they are not (attn_out depends on y_attn
 * through the projections and the attention), so a layer loop calls the ops
 * separately and this one-call form serves steps whose inputs are at hand together.
 * Batches of at most 512 tokens with 16-byte aligned buffers and whole-vector
 * rows run as ONE launch (the only dependency between the ops is the row-local
 * residual, so the launch holds independent row, token and SwiGLU jobs); larger
 * batches issue the five batched kernels. Results are the same either way (the
 * residual and the cache copies bit for bit). Every array is row-major and
 * contiguous: hidden, attn_out, y_attn, ffn_out, y_ffn [rows][dim]; q
 * [rows][num_q_heads][head_dim]; k, v [rows][num_kv_heads][head_dim]; gate, up,
 * act [rows][ffn]; caches [num_seqs][num_kv_heads][max_seq][head_dim];
 * positions and ids int32[rows]; seq_ids int32[rows] or NULL (all 0);
 * rope_table as for bm_rope_kv_store (NULL: fp64 angles from theta). Bad ids,
 * positions and sequences flag *d_status and skip that row's op, as the
 * separate calls do. */
typedef struct bm_layer_step {
  int64_t rows;
  int32_t dim, ffn;
  int64_t vocab;
  int32_t num_q_heads, num_kv_heads, head_dim, max_seq, num_seqs;
  float eps;
  double theta;
  const int32_t* ids;
  const void* embed;
  void* hidden;
  const void* attn_out;
  const void* w_attn;
  void* y_attn;
  void* q;
  const void* k;
  const void* v;
  const int32_t* positions;
  const int32_t* seq_ids;
  void* k_cache;
  void* v_cache;
  const void* rope_table;
  int32_t rope_table_len;
  const void* ffn_out;
  const void* w_ffn;
  void* y_ffn;
  const void* gate;
  const void* up;
  void* act;
} bm_layer_step_t;

int bm_layer_step(const bm_layer_step_t* step, bm_dtype_t dtype, int32_t* d_status, void* stream);

/* ---------------------------------------------------------------------------
 * RoPE table: fp32 (cos, sin) pairs laid out [max_pos][head_dim/2], entry
 * (p, i) for angle p / theta^(2i/head_dim), computed on the device in fp64
 * (the angle formula of the reference's CPU check loop,
 * tests/kernel_tests.cu:180, rounded once to fp32).
 * bm_rope_table_fill writes caller memory of max_pos*head_dim*4 bytes;
 * bm_rope_table_create allocates it (cudaMalloc) and fills it, synchronously.
 */
int bm_rope_table_fill(void* table, int32_t max_pos, int32_t head_dim,
                       double theta, void* stream);
int bm_rope_table_create(int32_t max_pos, int32_t head_dim, double theta,
                         void** table_out);
int bm_rope_table_destroy(void* table);

/* ---------------------------------------------------------------------------
 * Fused RoPE + KV-cache store for `rows` tokens.
 *   q [rows][num_q_heads][head_dim]  rotated in place;
 *   k [rows][num_kv_heads][head_dim] rotated and written to k_cache (k itself
 *                                    is not modified);
 *   v [rows][num_kv_heads][head_dim] copied to v_cache.
 * Caches are [num_seqs][num_kv_heads][max_seq][head_dim] (include/kv_cache.h:37-40).
 * Token r goes to sequence seq_ids[r] (all 0 when seq_ids is NULL) at position
 * positions[r] (pos0 + r when positions is NULL).
 * Rotation: the half-split pairing (i, i + head_dim/2) of launch_rope
 * (include/kernels.cuh:12-15, src/kernels.cu:126-140). Replaces the sequence
 * launch_rope + launch_kv_store(k) + launch_kv_store(v)
 * (src/execution_engine.cu:113-115; include/kernels.cuh:15,36).
 * rope_table from bm_rope_table_*, with table_len positions; NULL computes
 * cos/sin per pair on the device in fp64 from theta.
 */
int bm_rope_kv_store(void* q, const void* k, const void* v,
                     const int32_t* positions, int32_t pos0,
                     const int32_t* seq_ids,
                     void* k_cache, void* v_cache,
                     const void* rope_table, int32_t table_len, double theta,
                     int64_t rows, int32_t num_q_heads, int32_t num_kv_heads,
                     int32_t head_dim, int32_t max_seq, int32_t num_seqs,
                     bm_dtype_t dtype, int32_t* d_status, void* stream);

/* ---------------------------------------------------------------------------
 * RoPE in place on q [rows][num_q_heads][head_dim] and k [rows][num_kv_heads]
 * [head_dim] (either may be NULL with its head count 0). Batched launch_rope
 * (include/kernels.cuh:15, src/kernels.cu:126-148); positions/pos0,
 * rope_table/theta as in bm_rope_kv_store.
 */
int bm_rope(void* q, void* k, const int32_t* positions, int32_t pos0,
            const void* rope_table, int32_t table_len, double theta,
            int64_t rows, int32_t num_q_heads, int32_t num_kv_heads,
            int32_t head_dim, bm_dtype_t dtype, int32_t* d_status,
            void* stream);

/* ---------------------------------------------------------------------------
 * KV store: cache[seq][h][pos][:] = src[r][h][:] for `rows` tokens.
 * Batched launch_kv_store (include/kernels.cuh:36, src/kernels.cu:211-222);
 * positions/pos0 and seq_ids as in bm_rope_kv_store.
 */
int bm_kv_store(void* cache, const void* src, const int32_t* positions,
                int32_t pos0, const int32_t* seq_ids, int64_t rows,
                int32_t num_heads, int32_t head_dim, int32_t max_seq,
                int32_t num_seqs, bm_dtype_t dtype, int32_t* d_status,
                void* stream);

/* ---------------------------------------------------------------------------
 * Decode attention: one query token per entry of a batch, GQA.
 *   out[b][h][:] = softmax_j(q[b][h] . K[s][h/G][j] * scale) . V[s][h/G][j]
 * over positions j in [0, lens[b]) of cache sequence s = seq_ids[b] (0 when
 * seq_ids is NULL), G = num_q_heads / num_kv_heads (<= 16), scale <= 0 meaning
 * 1/sqrt(head_dim). q and out are [batch][num_q_heads][head_dim]; the caches are
 * [num_seqs][num_kv_heads][max_seq][head_dim] (bm_kv_cache_layer,
 * bm_rope_kv_store). lens is a device array; max_len is a host-side upper bound
 * of its entries that sizes the work split. head_dim <= 256 with whole 16-byte
 * rows. Replaces launch_attention (include/kernels.cuh:41,
 * src/kernels.cu:225-264: one token, heads = kv heads, three launches).
 * Long sequences are split across CTAs; the split results need
 * bm_decode_attention_workspace_size() bytes of device scratch, passed as
 * `workspace` (caller-owned; its contents need no initialisation). With less
 * scratch than that (or NULL) each (query, kv head) runs unsplit in one CTA:
 * same results, less parallelism. A query with an out-of-range sequence or a
 * length outside [1, max_len] (max_len <= max_seq) is skipped and flags
 * *d_status. */
int bm_decode_attention_workspace_size(int64_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                       int32_t head_dim, int32_t max_len, size_t* bytes_out);
int bm_decode_attention(void* out, const void* q, const void* k_cache, const void* v_cache,
                        const int32_t* seq_ids, const int32_t* lens, int32_t max_len, int64_t batch,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t max_seq,
                        int32_t num_seqs, float scale, void* workspace, size_t workspace_bytes,
                        bm_dtype_t dtype, int32_t* d_status, void* stream);

/* Decode attention with the new token's RoPE and K/V store in the same launch:
 * the engine's step for one token, launch_rope + launch_kv_store twice +
 * launch_attention (src/execution_engine.cu:113-116), equivalent to
 *   bm_rope_kv_store(q, k, v, positions, 0, seq_ids, k_cache, v_cache, rope_table, ...)
 *   bm_decode_attention(out, q, k_cache, v_cache, seq_ids, lens, ...)
 * for queries whose token sits at positions[b] < lens[b] of its own sequence (no
 * two queries of one call share a sequence). k and v are [batch][num_kv_heads]
 * [head_dim]; rope_table is required (bm_rope_table_*, rope_table_len positions).
 * On the CUDA-core path (head_dims other than 128) ONE launch: the CTA that attends
 * to the new position rotates k into the K cache, copies v into the V cache and
 * every CTA rotates its queries as it stages them, with the arithmetic of
 * bm_rope_kv_store. Head_dim 128 caches, read by TMA-fed kernels, take the two
 * calls. q is consumed: afterwards it holds its input or its rotation. On the
 * one-launch path a position outside [0, lens[b]) or past the table flags
 * BM_DEVERR_BAD_POSITION and that token is neither rotated nor stored (its query
 * attends over the cache as it is); the two-call path checks positions as
 * bm_rope_kv_store does. */
int bm_rope_kv_decode_attention(void* out, void* q, const void* k, const void* v, const int32_t* positions,
                                const void* rope_table, int32_t rope_table_len, const int32_t* seq_ids,
                                void* k_cache, void* v_cache, const int32_t* lens, int32_t max_len, int64_t batch,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t max_seq,
                                int32_t num_seqs, float scale, void* workspace, size_t workspace_bytes,
                                bm_dtype_t dtype, int32_t* d_status, void* stream);

/* Decode attention that allocates nothing, for callers that cannot call
 * cudaMalloc (a host application whose own arena owns all device memory, a
 * plugin in a process that reserved the GPU up front, a latency-critical path
 * that cannot afford cudaMalloc's implicit synchronisation). No counterpart in
 * the reference. Same arguments and results as bm_decode_attention, without the
 * workspace: the split partials live in an 8 MiB array compiled into the
 * library (one copy per GPU, held until the process exits). Arguments are
 * checked as bm_decode_attention checks them; then a batch whose split plan
 * (the one bm_decode_attention runs with a workspace of this array's size)
 * needs more than 8 MiB is rejected with BM_ERR_INVALID_ARGUMENT. The first
 * call in a CUDA context looks up that context's copy of the array (cached under
 * the context's unique id); make it before capturing any stream. All calls
 * share the array: calls that overlap on the GPU race on it and must be
 * serialised by the caller. */
int bm_decode_attention_static_scratch(void* out, const void* q, const void* k_cache, const void* v_cache,
                                       const int32_t* seq_ids, const int32_t* lens, int32_t max_len,
                                       int64_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                       int32_t head_dim, int32_t max_seq, int32_t num_seqs, float scale,
                                       bm_dtype_t dtype, int32_t* d_status, void* stream);

/* ---------------------------------------------------------------------------
 * Tensor-core GEMMs (tcgen05, bf16 operands, fp32 accumulation, bf16 output).
 * The activation is [rows][K] row-major; weights are [K][N] row-major, the
 * layout of launch_gemm's B operand (include/kernels.cuh:20, src/kernels.cu:83-121).
 * For BM_BF16: N and K multiples of 8, every pointer 16-byte aligned, any row
 * count (tcgen05). BM_F32 (any shape, no alignment needed) runs on CUDA cores in
 * fp32 (below).
 *
 * bm_gemm_swiglu: out[r][f] = silu(sum_d x[r][d] w_gate[d][f]) * sum_d x[r][d] w_up[d][f]
 * for x [rows][dim], w_gate and w_up [dim][hidden], out [rows][hidden]: the two
 * FFN input projections and the SwiGLU of src/execution_engine.cu:122-124 in one
 * kernel, the products kept in fp32 until the SwiGLU. bm_gemm: c[M][N] = a[M][K] b[K][N].
 * A pipeline wait that passes its time limit (a fault, never a slow input) sets
 * BM_DEVERR_TIMEOUT in *d_status.
 * BM_F32: fp32 arithmetic on CUDA cores, built for few rows (the reference
 * engine's one-token products, src/execution_engine.cu:81,110-125), K split over a
 * thread-block cluster and reduced in a fixed order (deterministic); d_status is
 * not used. bm_gemm_swiglu's fp32 SwiGLU is g / (1 + expf(-g)) * u, as bm_swiglu,
 * so it equals bm_gemm twice and bm_swiglu bit for bit.
 *
 * bm_gemm_shared_a: c[o] = a . b[o] for o < count (1 to 3), the products of one
 * activation with several weights (an attention block's Q, K and V projections):
 * c, b and n are host arrays of count device pointers and widths, a is [m][k],
 * b[o] [k][n[o]], c[o] [m][n[o]]. BM_F32 runs all of them in one launch; BM_BF16
 * runs bm_gemm once per product. */
int bm_gemm_swiglu(void* out, const void* x, const void* w_gate, const void* w_up, int64_t rows, int32_t dim,
                   int32_t hidden, bm_dtype_t dtype, int32_t* d_status, void* stream);
int bm_gemm(void* c, const void* a, const void* b, int64_t m, int32_t n, int32_t k, bm_dtype_t dtype,
            int32_t* d_status, void* stream);
int bm_gemm_shared_a(void* const* c, const void* a, const void* const* b, const int32_t* n, int32_t count,
                     int64_t m, int32_t k, bm_dtype_t dtype, int32_t* d_status, void* stream);

/* The RMSNorm before a projection and the projection together (the norms of
 * src/execution_engine.cu:80,109,121, after the residual adds of :118,126, each
 * followed by its products :81,110-112,122-123):
 *   x = h + d                      (d may be NULL: x = h)
 *   y = x * rsqrt(mean(x^2) + eps) * norm_weight       (as bm_rmsnorm computes it)
 *   swiglu == 0: c[o] = y . b[o] for o < count (1 to 3)   (as bm_gemm_shared_a)
 *   swiglu != 0: count 2, c[0] = silu(y . b[0]) * (y . b[1])   (as bm_gemm_swiglu)
 * h, d, residual_out and normed are [m][k]; b[o] is [k][n[o]]. residual_out
 * (may be NULL) receives x, the updated residual stream, when d is given; it must
 * not overlap h or d, which the kernel still reads while it is written.
 * BM_F32 with the normalised rows of a CTA's share of K fitting its shared memory
 * (one-token and few-token products): ONE launch, y never written to memory (its
 * sum of squares is ordered as the product kernel's threads hold the row, so y can
 * differ from bm_rmsnorm's in the last bit). Otherwise, and for BM_BF16, the norm
 * runs first into `normed` (scratch, always required), then the products. k > 0. */
int bm_rmsnorm_gemm(void* const* c, const void* h, const void* d, const void* norm_weight, float eps,
                    void* residual_out, void* normed, const void* const* b, const int32_t* n, int32_t count,
                    int32_t swiglu, int64_t m, int32_t k, bm_dtype_t dtype, int32_t* d_status, void* stream);

/* Softmax in place over num_vectors vectors of `size` elements, `stride`
 * elements apart (the gaps untouched): x = exp(x - max) / sum exp(x - max), fp32
 * arithmetic. Replaces launch_softmax(_batch) (include/kernels.cuh:23-26,
 * src/kernels.cu:150-180). */
int bm_softmax(void* x, int64_t size, int64_t num_vectors, int64_t stride, bm_dtype_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Batch-aware static KV cache. Replaces the reference's KVCache
 * (include/kv_cache.h:10-40, src/kv_cache.cu:4-47), which allocates
 * [max_batch][kv_heads][max_seq][head_dim] fp32 per layer but keeps one
 * current_seq_pos_ for the whole cache (src/kv_cache.cu:38-47). Here every
 * sequence has its own length, and the cache stores fp32 or bf16.
 *
 * bm_kv_cache_create allocates, per layer, one K and one V buffer of
 * num_seqs * num_kv_heads * max_seq * head_dim elements (cudaMalloc, zeroed) on
 * the current device, plus two int32 device arrays of max_tokens entries for the
 * positions and sequence ids of one batch. bm_kv_cache_append takes the
 * sequence id of each of `rows` new tokens (host array), gives each token the
 * next position of its sequence (tokens of one sequence in the order given),
 * copies positions and sequence ids to the device arrays on `stream`, and
 * returns their device pointers for bm_rope_kv_store. It fails, changing
 * nothing, if a sequence would pass max_seq or rows exceeds max_tokens.
 * The host copy is synchronous with respect to the host buffer (the call
 * returns after the upload is queued from the cache's own pinned staging).
 * Every append overwrites the same two device arrays, so issue each append and
 * the bm_rope_kv_store calls that read its arrays on one stream: stream order
 * then keeps the next append's upload behind the previous step's readers. */
typedef struct bm_kv_cache bm_kv_cache_t;

int bm_kv_cache_create(int32_t num_layers, int32_t num_seqs, int32_t num_kv_heads, int32_t max_seq,
                       int32_t head_dim, int32_t max_tokens, bm_dtype_t dtype, bm_kv_cache_t** cache_out);
int bm_kv_cache_destroy(bm_kv_cache_t* cache);
/* Device pointers of layer `layer`'s K and V caches, [num_seqs][kv_heads][max_seq][head_dim]. */
int bm_kv_cache_layer(const bm_kv_cache_t* cache, int32_t layer, void** keys, void** values);
/* Current length (next position) of sequence `seq`. */
int bm_kv_cache_seq_len(const bm_kv_cache_t* cache, int32_t seq, int32_t* len_out);
/* Starts sequence `seq` over (length 0); seq = -1 resets every sequence. */
int bm_kv_cache_reset(bm_kv_cache_t* cache, int32_t seq);
int bm_kv_cache_append(bm_kv_cache_t* cache, const int32_t* seq_ids, int64_t rows,
                       const int32_t** positions_dev, const int32_t** seq_ids_dev, void* stream);

/* Self-test of the bounded waits behind BM_DEVERR_TIMEOUT (the tensor-core
 * kernels' mbarrier waits): one CTA waits on a barrier that nothing completes,
 * with a limit of limit_ns in [1 ms, 2 s]. The wait gives up, ORs
 * BM_DEVERR_TIMEOUT into *d_status and the kernel finishes; the context stays
 * usable. d_result (device, 4 x int64): [0] 1 if the wait reported success
 * (expected 0), [1] its duration in ns (about limit_ns), [2] and [3] the same for
 * a second wait that honours the first one's abort (gives up at once). */
int bm_selftest_bounded_wait(int64_t limit_ns, int32_t* d_status, int64_t* d_result, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* BM_LAYER_OPS_H */
