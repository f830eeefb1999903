/*
 * dflash-b200 C ABI: the DFlash speculative draft/verify hot path on NVIDIA B200 (sm_100a).
 *
 * Every entry point is `extern "C"`, takes plain device pointers, element strides
 * and a cudaStream_t passed as `void*`, returns an int status (DFL_OK == 0) and
 * never synchronises the host. On a non-zero status dfl_last_error() returns a
 * message for the calling thread. bf16 buffers are passed as `void*`.
 *
 * The reference (Aryagm/dflash-mlx) is a Python/MLX package with no C ABI; each
 * entry point below names the reference call it replaces (path:line inside the
 * reference project). The Python host in dflash-mlx_b200/dflash_b200 binds these
 * with ctypes (dflash_b200/_lib.py lists every signature).
 */
#ifndef DFLASH_B200_H
#define DFLASH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DFL_ABI_VERSION 1

/* status codes */
#define DFL_OK 0
#define DFL_ERR_INVALID 1     /* null pointer, negative size, inconsistent arguments */
#define DFL_ERR_UNSUPPORTED 2 /* a shape / alignment this build has no kernel for */
#define DFL_ERR_CUDA 3        /* the CUDA launch itself failed */
#define DFL_ERR_WORKSPACE 4   /* caller-provided scratch is missing or too small */

/* GEMM epilogues (dfl_gemm_bf16) */
#define DFL_EPI_STORE 0    /* y = bf16(acc) */
#define DFL_EPI_RESIDUAL 1 /* y = bf16(residual + bf16(acc)); optional second copy to y2 (hidden-state tap) */
#define DFL_EPI_SILU_MUL 2 /* W rows packed per 64: [32 gate | 32 up]; y[:, n] = bf16(silu(gate) * up), N/2 columns */
#define DFL_EPI_ARGMAX 3   /* per row and 32 columns: (max bf16 logit, lowest index) into argmax partials */
#define DFL_EPI_STORE_F32 4 /* y = acc as fp32 (y is float*, ldy in floats): tensor-parallel partials */
#define DFL_EPI_PARTIALS 5  /* wide form only: the k_split fp32 K-range partials, unsummed, as slabs
                               y[s][M][N] (y float*, ldy must be N); with k_split 1 this is STORE_F32 */

/* keys per attention chunk: the fixed key ranges merged in order by dfl_attention */
#define DFL_ATTN_CHUNK 128

/* Per-sequence decode state kept on the device (64 bytes). */
typedef struct dfl_seq_state {
  int32_t start;      /* position of block[0]; the target KV cache holds positions [0, start) */
  int32_t pending;    /* verified rows of the tap buffer not yet in the draft cache */
  int32_t draft_len;  /* draft KV cache length */
  int32_t accepted;   /* acceptance length of the last step (matched + 1) */
  int32_t bonus;      /* posterior token committed after the accepted prefix */
  int32_t finished;   /* 1 once a stop token or the length limit has been committed */
  int32_t stop_index; /* index in the output of the first stop token, -1 if none */
  int32_t steps;      /* decode steps executed */
  int32_t total_max;  /* prompt length + max_new_tokens */
  int32_t prompt_len;
  int32_t reserved[6];
} dfl_seq_state;

int dfl_abi_version(void);
const char* dfl_last_error(void);

/* ---- dense projections ----------------------------------------------------
 * Y[M,N] = Xn[M,K] . W[N,K]^T with fp32 accumulation and a fused epilogue, where
 * Xn = X, or RMSNorm(X) * norm_w when norm_w != NULL (fused prologue: the row
 * sum of squares of X is given as sumsq_in[M][K/32] partials, one per 32
 * columns, summed in order; as written by DFL_EPI_STORE / DFL_EPI_RESIDUAL's
 * sumsq_out or by dfl_embed_bf16).
 * Replaces the nn.Linear (and the RMSNorm feeding it) of the verify / draft
 * forward: mlx-lm qwen3 Attention and MLP (driven from adapters.py:611-631),
 * DFlashAttention q/k/v/o projections (draft.py:75-98, 118-159), the draft fc
 * + hidden_norm (draft.py:196-201, 217) and lm_head_logits / lm_head_argmax
 * (adapters.py:264-271, 606-609; runtime.py:22-29 argmax).
 * K % 64 == 0, N % 32 == 0, x / w 16-byte aligned; the fused norm needs K <= 8192. Scratch: workspace of
 * dfl_gemm_workspace_bytes() bytes, zero-filled once before first use (the
 * kernel leaves its counters at zero); one workspace per stream.
 * DFL_EPI_ARGMAX writes float2 partials [M][dfl_gemm_argmax_tiles(N)] (one per
 * 32 columns). sumsq_out (nullable, STORE / RESIDUAL): per-row sum of squares of
 * the bf16 output per 32 columns, [M][N/32]. */
size_t dfl_gemm_workspace_bytes(int M, int N, int K, int epilogue);
int dfl_gemm_argmax_tiles(int N);

/* Weights are consumed in a pre-tiled HBM layout: W [N, K] row-major is cut into
 * 128-row x 64-column units, each stored as one contiguous 16 KB block in the
 * 128-byte-swizzled K-major image the tensor cores read (rows past N are zero),
 * units ordered by 128-row tile, then by k. dfl_pack_weight_bf16 converts a
 * row-major matrix (done once at load time). */
size_t dfl_packed_weight_bytes(int N, int K);
int dfl_pack_weight_bf16(const void* w, int N, int K, void* out, size_t out_bytes, void* stream);

int dfl_gemm_bf16(const void* x, int64_t ldx, const void* w_packed, int M, int N, int K, int epilogue,
                  const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                  void* argmax_partials, const void* norm_w, const float* sumsq_in, int n_parts, float eps,
                  float* sumsq_out, void* workspace, size_t workspace_bytes, void* stream);

/* Wide form of dfl_gemm_bf16 for many rows (batched verify: 4+ sequences x 16
 * rows), same arguments and epilogues plus k_split. Each 128-column x up-to-256-row
 * output tile runs its K loop in one tensor-core accumulator; k_split > 1 cuts K into
 * that many fixed contiguous ranges (fp32 partials summed in range order by a second
 * kernel, which then applies the epilogue), for weights with few 128-row tiles. A row's
 * result depends on K order and k_split only: identical for any M, but not
 * bit-identical to dfl_gemm_bf16's result, so runs compared bit for bit use one form
 * and one k_split. Compute-bound at large M. Workspace: dfl_gemm_wide_workspace_bytes
 * (RMSNorm prologue output when norm_w is given, split partials when k_split > 1). */
size_t dfl_gemm_wide_workspace_bytes(int M, int N, int K, int with_norm, int k_split);
int dfl_gemm_bf16_wide(const void* x, int64_t ldx, const void* w_packed, int M, int N, int K, int epilogue,
                       const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                       void* argmax_partials, const void* norm_w, const float* sumsq_in, int n_parts, float eps,
                       float* sumsq_out, int k_split, void* workspace, size_t workspace_bytes, void* stream);

/* ---- GEMM chain (decode blocks, M <= 16) --------------------------------------
 * Up to 6 dfl_gemm_bf16 calls, each usually reading the previous one's output, in one
 * persistent launch: the projections between two attention calls of a verify or draft
 * forward (o_proj -> gate/up -> down -> next layer's qkv; the same calls the reference's
 * mlx-lm qwen3 layers make, adapters.py:611-631, draft.py:173-187). Op k + 1 starts
 * streaming its weights while op k finishes; its X operand is read only after every CTA
 * completed op k. Arguments of each op as dfl_gemm_bf16 (1 <= M <= 16). A row's result
 * depends on N and K only (fixed unit ranges over a fixed grid), but is not
 * bit-identical to dfl_gemm_bf16's, so runs compared bit for bit use one form.
 * Workspace: dfl_gemm_chain_workspace_bytes, 256-byte aligned, zero-filled once (the
 * kernel leaves its counters at zero); one workspace per stream. */
typedef struct dfl_gemm_op {
  const void* x;
  int64_t ldx;
  const void* w_packed;
  int M, N, K, epilogue;
  const void* residual;
  int64_t ldr;
  void* y;
  int64_t ldy;
  void* y2;
  int64_t ldy2;
  void* argmax_partials;
  const void* norm_w;
  const float* sumsq_in;
  int n_parts;
  float eps;
  float* sumsq_out;
} dfl_gemm_op;
size_t dfl_gemm_chain_workspace_bytes(const dfl_gemm_op* ops, int n_ops);
int dfl_gemm_chain(const dfl_gemm_op* ops, int n_ops, void* workspace, size_t workspace_bytes, void* stream);

/* ---- tensor parallelism (Qwen3.5-27B, config 5) ------------------------------
 * Replaces the all-sum after the row-parallel projections of the reference's
 * sharded model (custom_qwen35_model.py:810 and shard_linear "sharded-to-all" at
 * :1338, :1347, :1375; sharding at :1286-1402). Buffers are peer-mapped with CUDA
 * IPC: dfl_tp_alloc (cudaMalloc + zero + 64-byte IPC handle), dfl_tp_open on the
 * other ranks, dfl_tp_close / dfl_tp_free to release.
 * dfl_tp_reduce_residual: parts[j] = rank j's n_slabs partial slabs [M, H] fp32 (row
 * stride H, slab_stride elements apart; DFL_EPI_STORE_F32 writes one, the wide
 * form's DFL_EPI_PARTIALS k_split) for this call; flags[j] = rank j's int flag
 * array (one slot per rank); epoch / done = this rank's call counter and CTA
 * counter (zeroed once). Sums the partials in rank then slab order in fp32 and writes
 * h <- bf16(h + bf16(sum)), tap (nullable) <- h, sumsq_out[M][H/32] (nullable).
 * Partial slots must alternate between two buffers on consecutive calls. A wait
 * that expires records device error 401. parts and flags are host arrays of n_ranks
 * device pointers (copied into the launch, so a captured graph keeps them). */
int dfl_tp_alloc(size_t bytes, void** ptr, unsigned char* ipc_handle_out);
int dfl_tp_open(const unsigned char* ipc_handle, void** ptr);
int dfl_tp_close(void* peer_ptr);
int dfl_tp_free(void* ptr);
int dfl_tp_reduce_residual(const void* const* parts, int* const* flags, int* epoch, int* done, int rank, int n_ranks,
                           int n_slabs, int64_t slab_stride, void* h, int64_t ldh, void* tap, int64_t ldtap,
                           float* sumsq_out, int M, int H, void* stream);
/* dfl_tp_reduce_residual that also writes xn = RMSNorm(h) * norm_w (row stride ldxn, the
 * input RMSNorm of the projection that follows: the reference's post_attention_layernorm /
 * next layer's input_layernorm after the all-reduce, custom_qwen35_model.py:810), each CTA
 * taking whole rows; the same bits as the GEMM's own norm from sumsq_out. H <= 8192. */
int dfl_tp_reduce_residual_norm(const void* const* parts, int* const* flags, int* epoch, int* done, int rank,
                                int n_ranks, int n_slabs, int64_t slab_stride, void* h, int64_t ldh, void* tap,
                                int64_t ldtap, float* sumsq_out, int M, int H, const void* norm_w, float eps, void* xn,
                                int64_t ldxn, void* stream);

/* Reads (and optionally clears) the device error record: non-zero when a kernel's
 * bounded wait gave up (the kernel returned instead of hanging). Synchronises
 * the given stream. */
int dfl_device_error(int* code, int clear, void* stream);

/* dfl_gemm_bf16 without a workspace argument, for callers that cannot allocate
 * device memory (host callbacks, plugins whose host owns every allocation,
 * engines that forbid cudaMalloc after start-up). No counterpart in the
 * reference. The split-K scratch is a fixed array inside this library
 * (dfl_gemm_noalloc_scratch_bytes(), about 5.4 MB held by every GPU that loads
 * the library until exit), sized for M <= 16 rows; larger M returns
 * DFL_ERR_UNSUPPORTED. No cudaMalloc / cudaFree is called. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture. All calls
 * share the array and each clears its counters first: calls that overlap on
 * the GPU (different streams, or concurrent host threads) race on it. */
size_t dfl_gemm_noalloc_scratch_bytes(void);
int dfl_gemm_bf16_noalloc(const void* x, int64_t ldx, const void* w_packed, int M, int N, int K, int epilogue,
                          const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                          void* argmax_partials, const void* norm_w, const float* sumsq_in, int n_parts, float eps,
                          float* sumsq_out, void* stream);

/* ---- row kernels ----------------------------------------------------------
 * RMSNorm y = w * x * rsqrt(mean(x^2) + eps) (fp32 math, bf16 out); w may be
 * NULL (unit weight). Replaces nn.RMSNorm / mx.fast.rms_norm (draft.py:167-171,
 * 198-201, 223; adapters.py:629). H % 256 == 0. */
int dfl_rmsnorm_bf16(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, int M, int H, float eps,
                     void* stream);

/* Token embedding gather (adapters.py:603-604 embed_tokens; runtime.py:410).
 * sumsq_out (nullable): per-row sum of squares per 32 columns, [M][H/32]
 * (feeds the fused RMSNorm prologue of dfl_gemm_bf16). */
int dfl_embed_bf16(const int32_t* tokens, const void* table, void* y, int64_t ldy, int M, int H, int V,
                   float* sumsq_out, void* stream);

/* q_norm / k_norm (per-head RMSNorm), non-interleaved RoPE over the first
 * rot_dim dims with inverse frequencies inv_freq[rot_dim/2], and the KV-cache
 * append at slot == pos[r] (rows with pos < 0 are skipped). Replaces the
 * q/k norm + rope + KVCache.update_and_fetch sequence of draft.py:118-147 and
 * of mlx-lm qwen3 Attention. Cache layout [seq][Hkv][cap][hd]. */
int dfl_qkv_rope_append(const void* qkv, int64_t ldqkv, int q_stride, const int32_t* pos, const int32_t* row_seq,
                        const void* q_norm, const void* k_norm, const float* inv_freq, void* q_out, void* k_cache,
                        void* v_cache, int64_t seq_stride, int64_t head_stride, int M, int Hq, int Hkv, int hd,
                        int rot_dim, float eps, int do_q, void* stream);

/* ---- attention ------------------------------------------------------------
 * GQA softmax(scale q.K^T) V over the cache. causal: row r sees keys
 * [0, pos[r]]; otherwise keys [0, kv_len[seq(r)]). Replaces
 * mx.fast.scaled_dot_product_attention at the verify (mask "causal",
 * adapters.py:620) and in DFlashAttention (draft.py:149-157). max_kv bounds
 * every row's key range (sizes the launch and the workspace). hd in {64, 128, 256}.
 * gate (nullable, row stride ldg, head h at h * gate_head_stride; 0 means hd):
 * out = bf16(attn) * bf16(sigmoid(gate)) per element,
 * the output gate of Qwen3.5 full attention (custom_qwen35_model.py:161-199).
 * seq_rows: with row_seq, each sequence's rows are contiguous runs of seq_rows
 * rows starting at multiples of seq_rows (a batched verify block); 0 = any
 * layout (slower launch). Rows of different sequences may share a 16-row tile;
 * a tile with more sequences than the layout allows sets device error 301.
 * key_chunk (multiple of 64; 0 = DFL_ATTN_CHUNK): keys per split; a row's result
 * depends on it, so runs to be compared bit for bit use the same value. One
 * chunk covering max_kv needs no workspace and no merge launch. */
size_t dfl_attention_workspace_bytes(int M, int Hq, int hd, int max_kv, int key_chunk);
int dfl_attention(const void* q, const void* k_cache, const void* v_cache, int64_t seq_stride, int64_t head_stride,
                  const int32_t* pos, const int32_t* row_seq, const int32_t* kv_len, int seq_rows, int M, int Hq, int Hkv, int hd,
                  int causal, float scale, int max_kv, int key_chunk, void* out, int64_t ldo, const void* gate, int64_t ldg,
                  int gate_head_stride, void* workspace, size_t workspace_bytes, void* stream);

/* Kernel launches one dfl_attention call of this shape makes (1: a single key chunk,
 * written directly; 2: chunk kernel + merge kernel), -1 for an unsupported shape. */
int dfl_attention_launches(int Hq, int Hkv, int hd, int max_kv, int key_chunk);

/* Paged KV caches (the same arithmetic, bit for bit, as the contiguous calls above).
 * The caches are pools of pages [n_pages][Hkv][page_size][hd] bf16 (page_stride and
 * head_stride in elements); page_table [seq][pt_stride] int32 maps sequence s's
 * positions [i * page_size, (i + 1) * page_size) to page page_table[s][i]. page_size is a
 * power of two >= 64. Every position a call reads or writes must have a page. A session
 * then reserves pages for each sequence's own length instead of the longest one's
 * (the reference grows one KVCache per layer per sequence, adapters.py:600-601; mlx-lm
 * KVCache.update_and_fetch / trim). */
int dfl_qkv_rope_append_paged(const void* qkv, int64_t ldqkv, int q_stride, const int32_t* pos, const int32_t* row_seq,
                              const void* q_norm, const void* k_norm, const float* inv_freq, void* q_out,
                              void* k_pages, void* v_pages, int64_t page_stride, int64_t head_stride,
                              const int32_t* page_table, int64_t pt_stride, int page_size, int M, int Hq, int Hkv,
                              int hd, int rot_dim, float eps, int do_q, void* stream);
/* The QKV projection of a decoder layer with the q/k head norm + RoPE + KV append fused
 * into it: dfl_gemm_bf16 (store epilogue; input RMSNorm prologue when norm_w is given)
 * writing the projection rows qkv [M][(Hq + 2 Hkv) * hd] (row stride ldqkv), then
 * dfl_qkv_rope_append over them (q_stride = rot_dim = hd, eps for the input norm and the
 * head norms, as Qwen3's rms_norm_eps), with the same bits as those two calls. For the
 * weight-streaming cluster form (M <= 16, head_dim 128: one output tile per head) the
 * append runs inside the GEMM launch after the tile's split-K reduction; otherwise the
 * two kernels run. page_table (nullable) as dfl_qkv_rope_append_paged. Replaces the
 * q/k/v projections + q_norm/k_norm + rope + KVCache.update_and_fetch of mlx-lm qwen3
 * Attention (driven from adapters.py:611-631) and of draft.py:118-147. */
int dfl_gemm_qkv_rope(const void* x, int64_t ldx, const void* w_packed, int M, int K, const void* norm_w,
                      const float* sumsq_in, int n_parts, float eps, void* qkv, int64_t ldqkv, const int32_t* pos,
                      const int32_t* row_seq, const void* q_norm, const void* k_norm, const float* inv_freq,
                      void* q_out, void* k_cache, void* v_cache, int64_t seq_stride, int64_t head_stride,
                      const int32_t* page_table, int64_t pt_stride, int page_size, int Hq, int Hkv, int hd,
                      void* workspace, size_t workspace_bytes, void* stream);
/* The draft's context rows (draft.py:118-147 for every DFlashDecoderLayer: k_proj / v_proj
 * of the context, k_norm, RoPE at the rows' positions, append to each layer's cache) for
 * n_layers layers at once: one GEMM over the stacked per-layer K/V weights
 * [n_layers * 2 * Hkv * hd, K] writing kv (layer l's columns at l * 2 * Hkv * hd), then layer
 * l's k_norm (k_norms[l], a host array of device pointers) + RoPE + append into
 * k_cache / v_cache + l * layer_stride elements. At M <= 16 rows and head_dim 128 the
 * appends run inside the GEMM launch; otherwise one append launch per layer follows. The
 * same bits as dfl_gemm_bf16 + dfl_qkv_rope_append(_paged) per layer (Hq = 0, do_q = 0).
 * n_layers <= 16. */
int dfl_gemm_kv_append_layers(const void* x, int64_t ldx, const void* w_packed, int M, int K, const void* norm_w,
                              const float* sumsq_in, int n_parts, float eps, void* kv, int64_t ldkv,
                              const int32_t* pos, const int32_t* row_seq, const void* const* k_norms,
                              const float* inv_freq, void* k_cache, void* v_cache, int64_t layer_stride,
                              int64_t seq_stride, int64_t head_stride, const int32_t* page_table, int64_t pt_stride,
                              int page_size, int n_layers, int Hkv, int hd, void* workspace, size_t workspace_bytes,
                              void* stream);

/* Kernel launches one dfl_gemm_qkv_rope call of this shape makes (1: the append inside the
 * GEMM launch; 2: GEMM + append kernel), -1 for a bad shape. With Hq = 0 and Hkv = n_layers x
 * the layer's kv heads it answers for dfl_gemm_kv_append_layers (1: fused; 2: GEMM + one
 * append launch per layer). */
int dfl_gemm_qkv_rope_launches(int M, int K, int Hq, int Hkv, int hd);
int dfl_attention_paged(const void* q, const void* k_pages, const void* v_pages, int64_t page_stride,
                        int64_t head_stride, const int32_t* page_table, int64_t pt_stride, int page_size,
                        const int32_t* pos, const int32_t* row_seq, const int32_t* kv_len, int seq_rows, int M, int Hq,
                        int Hkv, int hd, int causal, float scale, int max_kv, int key_chunk, void* out, int64_t ldo,
                        const void* gate, int64_t ldg, int gate_head_stride, void* workspace, size_t workspace_bytes,
                        void* stream);

/* dfl_qkv_rope_append followed by causal dfl_attention in one launch, for head_dim 128 with
 * rotary over the whole head (the Qwen3 verify block: mlx-lm qwen3 Attention's q/k norm,
 * RoPE, KVCache.update_and_fetch and scaled_dot_product_attention, adapters.py:611-631).
 * qkv: the raw projection rows [M][(Hq + 2 Hkv) * 128] (q heads, k heads, v heads). Each
 * row's key and value are normalised, rotated and written into the caches at pos[r] by the
 * CTA whose key range holds that position, which is the only CTA that reads them; the query
 * tile is normalised and rotated on load. Bit-identical to the two calls. Needs every
 * sequence's rows inside one 16-row tile: row_seq null with M <= 16, or seq_rows dividing
 * 16 (otherwise DFL_ERR_UNSUPPORTED). Workspace as dfl_attention_workspace_bytes(M, Hq,
 * 128, max_kv, key_chunk). */
int dfl_attention_qkv(const void* qkv, int64_t ldqkv, const void* q_norm, const void* k_norm, const float* inv_freq,
                      float eps, void* k_cache, void* v_cache, int64_t seq_stride, int64_t head_stride,
                      const int32_t* pos, const int32_t* row_seq, int seq_rows, int M, int Hq, int Hkv, float scale,
                      int max_kv, int key_chunk, void* out, int64_t ldo, void* workspace, size_t workspace_bytes,
                      void* stream);

/* ---- speculative step control ---------------------------------------------
 * Greedy argmax from DFL_EPI_ARGMAX partials (runtime.py:22-29 at temperature 0). */
int dfl_argmax_reduce(const void* partials, int M, int n_tiles, int32_t* out, void* stream);

/* Temperature sampling (sample_tokens, runtime.py:22-29, at temperature >= 1e-5) by
 * Gumbel-max. dfl_sample_keys: key of row b * bs + i = a mix of (seed, tag, b,
 * state[b].start + i + offset) -- the absolute position the row predicts (offset 1 for
 * verify rows, 0 for draft rows), so plain and speculative decoding draw the same noise
 * for the same position. dfl_sample_partials: for each row of bf16 logits [M, V] (row
 * stride ld) and each 32 columns, (max of bf16(logit) * inv_temperature +
 * Gumbel(key[row], column), lowest index) in the DFL_EPI_ARGMAX partial layout. */
int dfl_sample_keys(const dfl_seq_state* state, int B, int bs, uint64_t seed, int tag, int offset, uint64_t* keys,
                    void* stream);
int dfl_sample_partials(const void* logits, int64_t ld, int M, int V, const uint64_t* keys, float inv_temperature,
                        void* partials, void* stream);

/* Builds block = [out[start], mask_id x (bs-1)] (runtime.py:408) and the
 * verify / draft positions for every sequence. */
int dfl_step_prepare(dfl_seq_state* state, const int32_t* out_tokens, int64_t out_stride, int32_t* block, int bs,
                     int mask_id, int32_t* target_pos, int32_t* draft_ctx_pos, int32_t* draft_block_pos,
                     int32_t* draft_kv_len, int B, void* stream);

/* block[1:] = draft argmax (runtime.py:417-423), or injected tokens when
 * inject_tokens != NULL; then trims the draft cache back to its context
 * (trim_draft_cache, runtime.py:32-34, 420). */
int dfl_draft_commit(dfl_seq_state* state, const void* partials, int n_tiles, int32_t* block, int bs,
                     const int32_t* inject_tokens, int64_t inject_stride, const int32_t* inject_len,
                     int64_t inject_len_stride, const int32_t* inject_noise, int64_t noise_stride, int B,
                     void* stream);

/* Posterior argmax, longest_prefix_match (runtime.py:41-47), accepted =
 * matched + 1 and bonus token (runtime.py:139-163), commit and stop / length
 * checks (runtime.py:488-507); the KV rollback of rewind_kv_caches
 * (adapters.py:697-700) is the length update state.start += accepted. */
int dfl_verify_accept(dfl_seq_state* state, const void* partials, int n_tiles, const int32_t* block, int bs,
                      int32_t* out_tokens, int64_t out_stride, int32_t* posterior, const int32_t* stop_ids,
                      int n_stop, int32_t* accept_log, int64_t log_stride, int B, void* stream);

/* ---- gated-delta-net layer (Qwen3.5 linear attention) ------------------------
 * dfl_gdn_prep: from the in-projection rows proj [B*T][ldp] = [qkv (C = 2*Hk*Dk + Hv*Dv)
 * | z (Hv*Dv) | b (Hv) | a (Hv)] and the conv state [B][3][C]: depthwise conv1d (k=4)
 * + SiLU, q <- Dk^-1 * rmsnorm(q), k <- Dk^-1/2 * rmsnorm(k), beta = sigmoid(b),
 * g = exp(-exp(A_log) * softplus(a + dt_bias)); window (nullable; win_stride elements
 * per sequence, 0 = packed 3+T rows) keeps
 * [conv state | qkv] for the rollback. Replaces custom_qwen35_model.py:409-450. */
int dfl_gdn_prep(const void* proj, int64_t ldp, const void* conv_w, const float* A_log, const float* dt_bias,
                 const void* conv_state, void* window, int64_t win_stride, void* q, void* k, void* v, float* g,
                 float* beta, int B, int T, int Hk, int Hv, int Dk, int Dv, float eps, void* stream);

/* Rollback to "after accepted[b * acc_stride] tokens" of the block: state[b] <-
 * snapshots[b][acc-1] (when snapshots != NULL), conv_state[b] <- window[b][acc..acc+2]
 * (when window != NULL). Replaces rollback_linear_caches (custom_qwen35_model.py:1029-1074,
 * adapters.py:510-560), which replays the recurrence instead. */
int dfl_gdn_rollback(float* state, const float* snapshots, void* conv_state, const void* window,
                     int64_t win_stride, const int32_t* accepted, int acc_stride, int B, int T, int Hv, int Dv,
                     int Dk, int C, void* stream);

/* RMSNormGated per value head: out = bf16(w * rmsnorm(o)) * bf16(silu(z)) (adapters.py:226-227). */
int dfl_gated_rmsnorm(const void* o, int64_t ldo, const void* z, int64_t ldz, const void* w, void* out, int64_t ldout,
                      int M, int H, int D, float eps, void* stream);

/* ---- gated-delta recurrence -----------------------------------------------
 * q,k [B,T,Hk,Dk] bf16, v [B,T,Hv,Dv] bf16, g (decay multiplier) and beta
 * [B,T,Hv] fp32, state [.,Hv,Dv,Dk] fp32. Writes o [B,T,Hv,Dv] bf16 (nullable),
 * the state after every token into snapshots [B,T,Hv,Dv,Dk] (nullable) and
 * the final state (nullable; may alias state_in). state_slot (nullable)
 * selects snapshot slot[b] of state_in (zero-copy rollback). tokens (nullable):
 * sequence b advances over its first min(T, tokens[b * tokens_stride]) tokens only
 * (the accepted prefix of a verify block, read on the device). Replaces mlx-lm
 * gated_delta_kernel / gated_delta_ops (custom_qwen35_model.py:452-476) and,
 * with o and snapshots NULL and tokens = the accepted lengths,
 * advance_gated_delta_states (adapters.py:93-135, the replay of
 * rollback_linear_caches, adapters.py:505-560). */
int dfl_gdr_recurrence(const void* q, const void* k, const void* v, const float* g, const float* beta,
                       const float* state_in, int64_t state_in_bstride, const int32_t* state_slot, float* state_out,
                       float* snapshots, void* o, int B, int T, int Hk, int Hv, int Dk, int Dv, const int32_t* tokens,
                       int tokens_stride, void* stream);

/* ---- step-level driver (the decode loop body from C) ------------------------
 * Replaces the loop body of dflash_generate_stream (runtime.py:406-518) for hosts
 * that are not Python: dfl_draft_step = block [last, mask x (bs-1)], draft forward over
 * the new taps and the block, proposals (runtime.py:407-423, draft.py:109-223);
 * dfl_verify_step = target verify forward with taps, greedy argmax, longest-prefix
 * accept, bonus, commit and stop / length checks (runtime.py:117-163, 488-507,
 * adapters.py:611-631), writing accepted / bonus / finished into the device state;
 * dfl_rollback = the cache rollback (rewind_kv_caches, adapters.py:697-700; for the dense
 * family the accept has already moved the cache length, so it only validates).
 * Dense Qwen3 family. The context borrows the weights (device pointers, GEMM weights
 * packed by dfl_pack_weight_bf16; the caller keeps them alive) and allocates every
 * session buffer in dfl_ctx_create; the step calls allocate nothing and do not sync
 * the host. Unless DFL_CTX_NO_GRAPH is set, the first call of each half records it as
 * a CUDA graph on a private stream (later calls launch the graph on `stream`); call
 * dfl_ctx_set_injection before the first step or the draft half is recorded again. */
typedef struct dfl_layer_weights {
  const void* in_norm;   /* [H] bf16 input_layernorm */
  const void* post_norm; /* [H] bf16 post_attention_layernorm */
  const void* w_qkv;     /* packed [(Hq + 2 Hkv) hd, H]: q_proj, k_proj, v_proj rows */
  const void* w_o;       /* packed [H, Hq hd] */
  const void* w_gu;      /* packed [2F, H], gate / up interleaved per 64 rows (32 | 32) */
  const void* w_down;    /* packed [H, F] */
  const void* q_norm;    /* [hd] bf16 */
  const void* k_norm;    /* [hd] bf16 */
} dfl_layer_weights;

typedef struct dfl_qwen3_desc {
  int hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab, rope_dim;
  float eps, rope_theta;
  const void* embed;      /* [V, H] bf16 row-major (embedding gather) */
  const void* lm_head;    /* packed [V, H] (the embedding again when tied) */
  const void* final_norm; /* [H] bf16 */
  const dfl_layer_weights* layers; /* n_layers entries (copied at create) */
} dfl_qwen3_desc;

typedef struct dfl_draft_desc {
  int hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, block_size, mask_token_id, n_taps, causal;
  float eps, rope_theta;
  const int32_t* target_layer_ids; /* host, n_taps ascending (copied at create) */
  const void* fc;                  /* packed [H, n_taps H] */
  const void* hidden_norm;         /* [H] bf16 */
  const void* final_norm;          /* [H] bf16 */
  const void* w_ctx_kv;            /* packed [n_layers 2 Hkv hd, H]: every layer's k_proj then v_proj rows */
  const dfl_layer_weights* layers; /* n_layers entries (copied at create) */
} dfl_draft_desc;

typedef struct dfl_ctx dfl_ctx;
#define DFL_CTX_NO_GRAPH 1

int dfl_ctx_create(const dfl_qwen3_desc* target, const dfl_draft_desc* draft, int batch, int max_total,
                   int block_size, const int32_t* stop_ids, int n_stop, int max_steps, int flags, dfl_ctx** out);
int dfl_ctx_destroy(dfl_ctx* ctx);
/* Prefill of sequence `seq` from host tokens (chunks of 128 rows, taps into the draft
 * cache) and its first greedy token (runtime.py:383-404). A set-up call: it synchronises. */
int dfl_ctx_prefill(dfl_ctx* ctx, int seq, const int32_t* tokens, int n_tokens, int max_new_tokens, void* stream);
/* Oracle-injected drafts (benchmarks): block[1 + i] = trace[b][start + 1 + i] for
 * i < lengths[b][step], else noise[b][step * bs + i] (device arrays; NULL trace = off). */
int dfl_ctx_set_injection(dfl_ctx* ctx, const int32_t* trace, int64_t trace_stride, const int32_t* lengths,
                          int64_t lengths_stride, const int32_t* noise, int64_t noise_stride);
int dfl_draft_step(dfl_ctx* ctx, void* stream);
int dfl_verify_step(dfl_ctx* ctx, void* stream);
int dfl_rollback(dfl_ctx* ctx, void* stream);
/* Device pointers of the state [B], output tokens [B][out_stride] and acceptance log
 * [B][log_stride] (for device-side consumers), and a synchronous host copy of them. */
int dfl_ctx_buffers(dfl_ctx* ctx, dfl_seq_state** state, int32_t** out_tokens, int64_t* out_stride,
                    int32_t** accept_log, int64_t* log_stride);
int dfl_ctx_read(dfl_ctx* ctx, dfl_seq_state* state, int32_t* out_tokens, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DFLASH_B200_H */
