// Step-level C ABI: one speculative DFlash step driven from C, for hosts that are not
// Python. It replaces the loop body of the reference's dflash_generate_stream
// (dflash_mlx/runtime.py:406-518): the draft proposal (runtime.py:407-423, draft.py:109-223),
// the parallel-replay verify with taps, argmax, longest-prefix accept and bonus
// (runtime.py:117-163, adapters.py:611-631) and the KV rollback (adapters.py:697-700).
//
// A context borrows the caller's weights (device pointers; GEMM weights in the packed
// layout of dfl_pack_weight_bf16) and owns everything a session needs: per-sequence step
// state, output tokens, KV caches of target and draft, the tap buffer, activations and
// kernel scratch. All of it is allocated in dfl_ctx_create; the step calls allocate
// nothing and never synchronise the host. The launch sequence per step is the one the
// Python runtime issues (dflash_b200/model.py, runtime.py), argument for argument, so the
// two drivers commit the same tokens bit for bit. The first step records the draft half
// and the verify half as two CUDA graphs on a private stream; later steps launch them on
// the caller's stream.
//
// Scope: the dense Qwen3 family (benchmark configurations 1, 3 and 4). The Qwen3.5
// hybrid is driven from the Python host (dflash_b200/hybrid.py).
#include "common.cuh"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace {

using dfl::set_error;

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
};

struct Ctx {
  dfl_qwen3_desc t{};
  dfl_draft_desc d{};
  bool has_draft = false;
  std::vector<dfl_layer_weights> tl, dl;
  std::vector<int> tap_ids;
  int B = 0, bs = 0, cap = 0, max_rows = 0;
  bool batched = false;
  int key_chunk = 128;
  int wide_split_max = 1;
  int n_sm = 148;
  int n_stop = 0;
  int max_steps = 0;
  std::vector<DevBuf> owned;
  // device buffers
  dfl_seq_state* state = nullptr;
  int* out_tokens = nullptr;  // [B][cap]
  int* block = nullptr;       // [B*bs]
  int* tpos = nullptr;
  int* dpos_ctx = nullptr;
  int* dpos_blk = nullptr;
  int* dkv_len = nullptr;
  int* row_seq = nullptr;     // [max_rows] (row / bs, or the prefill sequence)
  int* accept_log = nullptr;  // [B][max_steps]
  int* stop_ids = nullptr;
  int* prefill_tok = nullptr;
  int* prefill_pos = nullptr;
  int* first_tok = nullptr;
  __nv_bfloat16 *tk = nullptr, *tv = nullptr, *dk = nullptr, *dv = nullptr;  // [L][B][Hkv][cap][hd]
  __nv_bfloat16* taps = nullptr;                                            // [max_rows][ntaps*H]
  float* t_inv_freq = nullptr;
  float* d_inv_freq = nullptr;
  // target activations
  __nv_bfloat16 *h = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
  float *ss = nullptr, *argmax = nullptr;
  // draft activations
  __nv_bfloat16 *dh = nullptr, *dqkv = nullptr, *dq = nullptr, *dattn = nullptr, *dact = nullptr;
  __nv_bfloat16 *dfc = nullptr, *dkvp = nullptr;
  float *dss = nullptr, *dss_ctx = nullptr, *dargmax = nullptr;
  // scratch
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  void* wide_ws = nullptr;
  size_t wide_ws_bytes = 0;
  void* attn_ws = nullptr;
  size_t attn_ws_bytes = 0;
  void* chain_ws = nullptr;
  size_t chain_ws_bytes = 0;
  bool use_chain = true;
  // inject
  const int *inj_tok = nullptr, *inj_len = nullptr, *inj_noise = nullptr;
  int64_t inj_tok_stride = 0, inj_len_stride = 0, inj_noise_stride = 0;
  // graphs
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t g_draft = nullptr, g_verify = nullptr;
  bool use_graph = true;
};

int fail_cuda(const char* what, cudaError_t e) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return DFL_ERR_CUDA;
}

template <class T>
int alloc(Ctx* c, T** out, size_t n, bool zero = true) {
  void* p = nullptr;
  const size_t bytes = n * sizeof(T) > 0 ? n * sizeof(T) : 16;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail_cuda("dfl_ctx_create: cudaMalloc", e);
  c->owned.push_back({p, bytes});
  if (zero && (e = cudaMemset(p, 0, bytes)) != cudaSuccess) return fail_cuda("dfl_ctx_create: cudaMemset", e);
  *out = static_cast<T*>(p);
  return DFL_OK;
}

#define TRY(x)                  \
  do {                          \
    const int _s = (x);         \
    if (_s != DFL_OK) return _s; \
  } while (0)

int wide_split(const Ctx* c, int N, int K) {
  if (c->wide_split_max <= 1) return 1;
  const int n_tiles = (N + 127) / 128;
  // round(n_sm / n_tiles) with ties to even, as Python's round()
  const double r = (double)c->n_sm / n_tiles;
  double fl = std::floor(r);
  long long rr = (long long)fl;
  const double frac = r - fl;
  if (frac > 0.5 || (frac == 0.5 && (rr & 1))) ++rr;
  long long v = rr < c->wide_split_max ? rr : c->wide_split_max;
  if (v > K / 64) v = K / 64;
  return v < 1 ? 1 : (int)v;
}

int gemm(Ctx* c, const void* x, int64_t ldx, const void* w, int M, int N, int K, int epi, const void* res,
         int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2, void* part, const void* norm_w,
         const float* ss_in, float* ss_out, float eps, cudaStream_t s) {
  const int n_parts = norm_w ? K / 32 : 0;
  if (c->batched)
    return dfl_gemm_bf16_wide(x, ldx, w, M, N, K, epi, res, ldr, y, ldy, y2, ldy2, part, norm_w, ss_in, n_parts,
                              eps, ss_out, wide_split(c, N, K), c->wide_ws, c->wide_ws_bytes, s);
  return dfl_gemm_bf16(x, ldx, w, M, N, K, epi, res, ldr, y, ldy, y2, ldy2, part, norm_w, ss_in, n_parts, eps,
                       ss_out, c->gemm_ws, c->gemm_ws_bytes, s);
}

size_t kv_layer_elems(const Ctx* c, int hkv, int hd) { return (size_t)c->B * hkv * c->cap * hd; }

// The QKV projection (input RMSNorm fused) and the q/k head norm + RoPE + cache append of
// one decoder layer: one dfl_gemm_qkv_rope call on the M <= 16 GEMM forms unless
// DFLASH_B200_FUSED_QKV_ROPE=0 (the Python host's model.qkv_rope_ok rule), else the two
// calls; both give the same bits.
bool fused_qkv_rope(const Ctx* c, int hd, int rot_dim) {
  static const bool off = [] {
    const char* e = std::getenv("DFLASH_B200_FUSED_QKV_ROPE");
    return e && e[0] == '0';
  }();
  return !off && !c->batched && rot_dim == hd;
}

int qkv_rope(Ctx* c, const void* x, const float* ss, int H, const dfl_layer_weights& w, int M, int Hq, int Hkv, int hd,
             int rot_dim, float eps, const int* pos, const int* row_seq, const float* inv_freq, void* qkv, void* q,
             __nv_bfloat16* kc, __nv_bfloat16* vc, cudaStream_t s) {
  const int nqkv = (Hq + 2 * Hkv) * hd;
  if (fused_qkv_rope(c, hd, rot_dim))
    return dfl_gemm_qkv_rope(x, H, w.w_qkv, M, H, w.in_norm, ss, H / 32, eps, qkv, nqkv, pos, row_seq, w.q_norm,
                             w.k_norm, inv_freq, q, kc, vc, (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, nullptr, 0, 0, Hq, Hkv, hd,
                             c->gemm_ws, c->gemm_ws_bytes, s);
  TRY(gemm(c, x, H, w.w_qkv, M, nqkv, H, DFL_EPI_STORE, nullptr, 0, qkv, nqkv, nullptr, 0, nullptr, w.in_norm, ss,
           nullptr, eps, s));
  return dfl_qkv_rope_append(qkv, nqkv, hd, pos, row_seq, w.q_norm, w.k_norm, inv_freq, q, kc, vc,
                             (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, M, Hq, Hkv, hd, rot_dim, eps, 1, s);
}

// One dfl_gemm_op (the arguments of gemm() above).
dfl_gemm_op gop(const void* x, int64_t ldx, const void* w, int M, int N, int K, int epi, const void* res, int64_t ldr,
                void* y, int64_t ldy, void* y2, int64_t ldy2, void* part, const void* norm_w, const float* ss_in,
                float* ss_out, float eps) {
  dfl_gemm_op o;
  o.x = x;
  o.ldx = ldx;
  o.w_packed = w;
  o.M = M;
  o.N = N;
  o.K = K;
  o.epilogue = epi;
  o.residual = res;
  o.ldr = ldr;
  o.y = y;
  o.ldy = ldy;
  o.y2 = y2;
  o.ldy2 = ldy2;
  o.argmax_partials = part;
  o.norm_w = norm_w;
  o.sumsq_in = ss_in;
  o.n_parts = norm_w ? K / 32 : 0;
  o.eps = eps;
  o.sumsq_out = ss_out;
  return o;
}

// Whether a forward over M rows runs its projections as GEMM chains (the Python host's
// rule, model.chain_ok: decode blocks of the one-sequence kernel forms).
bool chain_ok(const Ctx* c, int M) { return c->use_chain && M <= 16 && !c->batched; }

int run_chain(Ctx* c, std::vector<dfl_gemm_op>& ops, cudaStream_t s) {
  if (ops.empty()) return DFL_OK;
  const int st = dfl_gemm_chain(ops.data(), (int)ops.size(), c->chain_ws, c->chain_ws_bytes, s);
  ops.clear();
  return st;
}

// Target block forward over M rows (tokens / pos device arrays): taps into `taps` (row
// stride ntaps*H), lm_head argmax partials into c->argmax. Mirrors TargetModel.forward.
int target_forward(Ctx* c, const int* tokens, const int* pos, int M, const int* row_seq, int seq_rows,
                   int max_kv, __nv_bfloat16* taps, cudaStream_t s) {
  const dfl_qwen3_desc& t = c->t;
  const int H = t.hidden, hd = t.head_dim, Hq = t.n_heads, Hkv = t.n_kv_heads;
  const int ntaps = (int)c->tap_ids.size();
  const int nqkv = (Hq + 2 * Hkv) * hd;
  const float eps = t.eps;
  TRY(dfl_embed_bf16(tokens, t.embed, c->h, H, M, H, t.vocab, c->ss, s));
  if (chain_ok(c, M)) {
    std::vector<dfl_gemm_op> ops;
    if (t.n_layers > 0)
      ops.push_back(gop(c->h, H, c->tl[0].w_qkv, M, nqkv, H, DFL_EPI_STORE, nullptr, 0, c->qkv, nqkv, nullptr, 0,
                        nullptr, c->tl[0].in_norm, c->ss, nullptr, eps));
    for (int l = 0; l < t.n_layers; ++l) {
      const dfl_layer_weights& w = c->tl[l];
      TRY(run_chain(c, ops, s));
      __nv_bfloat16* kc = c->tk + (size_t)l * kv_layer_elems(c, Hkv, hd);
      __nv_bfloat16* vc = c->tv + (size_t)l * kv_layer_elems(c, Hkv, hd);
      TRY(dfl_qkv_rope_append(c->qkv, nqkv, hd, pos, row_seq, w.q_norm, w.k_norm, c->t_inv_freq, c->q, kc, vc,
                              (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, M, Hq, Hkv, hd, t.rope_dim, eps, 1,
                              s));
      TRY(dfl_attention(c->q, kc, vc, (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, pos, row_seq, nullptr,
                        seq_rows, M, Hq, Hkv, hd, 1, (float)(1.0 / std::sqrt((double)hd)), max_kv, c->key_chunk,
                        c->attn, Hq * hd, nullptr, 0, 0, c->attn_ws, c->attn_ws_bytes, s));
      void* tap = nullptr;
      for (int i = 0; i < ntaps; ++i)
        if (c->tap_ids[i] == l && taps) tap = taps + (size_t)i * H;
      ops.push_back(gop(c->attn, Hq * hd, w.w_o, M, H, Hq * hd, DFL_EPI_RESIDUAL, c->h, H, c->h, H, nullptr, 0,
                        nullptr, nullptr, nullptr, c->ss, eps));
      ops.push_back(gop(c->h, H, w.w_gu, M, 2 * t.ffn, H, DFL_EPI_SILU_MUL, nullptr, 0, c->act, t.ffn, nullptr, 0,
                        nullptr, w.post_norm, c->ss, nullptr, eps));
      ops.push_back(gop(c->act, t.ffn, w.w_down, M, H, t.ffn, DFL_EPI_RESIDUAL, c->h, H, c->h, H, tap,
                        tap ? (int64_t)ntaps * H : 0, nullptr, nullptr, nullptr, c->ss, eps));
      if (l + 1 < t.n_layers)
        ops.push_back(gop(c->h, H, c->tl[l + 1].w_qkv, M, nqkv, H, DFL_EPI_STORE, nullptr, 0, c->qkv, nqkv, nullptr,
                          0, nullptr, c->tl[l + 1].in_norm, c->ss, nullptr, eps));
    }
    ops.push_back(gop(c->h, H, t.lm_head, M, t.vocab, H, DFL_EPI_ARGMAX, nullptr, 0, nullptr, 0, nullptr, 0,
                      c->argmax, t.final_norm, c->ss, nullptr, eps));
    return run_chain(c, ops, s);
  }
  for (int l = 0; l < t.n_layers; ++l) {
    const dfl_layer_weights& w = c->tl[l];
    __nv_bfloat16* kc = c->tk + (size_t)l * kv_layer_elems(c, Hkv, hd);
    __nv_bfloat16* vc = c->tv + (size_t)l * kv_layer_elems(c, Hkv, hd);
    TRY(qkv_rope(c, c->h, c->ss, H, w, M, Hq, Hkv, hd, t.rope_dim, eps, pos, row_seq, c->t_inv_freq, c->qkv, c->q,
                 kc, vc, s));
    TRY(dfl_attention(c->q, kc, vc, (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, pos, row_seq, nullptr,
                      seq_rows, M, Hq, Hkv, hd, 1, (float)(1.0 / std::sqrt((double)hd)), max_kv, c->key_chunk, c->attn,
                      Hq * hd, nullptr, 0, 0, c->attn_ws, c->attn_ws_bytes, s));
    TRY(gemm(c, c->attn, Hq * hd, w.w_o, M, H, Hq * hd, DFL_EPI_RESIDUAL, c->h, H, c->h, H, nullptr, 0, nullptr,
             nullptr, nullptr, c->ss, eps, s));
    TRY(gemm(c, c->h, H, w.w_gu, M, 2 * t.ffn, H, DFL_EPI_SILU_MUL, nullptr, 0, c->act, t.ffn, nullptr, 0, nullptr,
             w.post_norm, c->ss, nullptr, eps, s));
    void* tap = nullptr;
    for (int i = 0; i < ntaps; ++i)
      if (c->tap_ids[i] == l && taps) tap = taps + (size_t)i * H;
    TRY(gemm(c, c->act, t.ffn, w.w_down, M, H, t.ffn, DFL_EPI_RESIDUAL, c->h, H, c->h, H, tap,
             tap ? (int64_t)ntaps * H : 0, nullptr, nullptr, nullptr, c->ss, eps, s));
  }
  return gemm(c, c->h, H, t.lm_head, M, t.vocab, H, DFL_EPI_ARGMAX, nullptr, 0, nullptr, 0, nullptr, 0, c->argmax,
              t.final_norm, c->ss, nullptr, eps, s);
}

// hidden_norm(fc(taps)) and every draft layer's K/V of those rows into the draft cache
// (DraftModel.ingest_context; rows with pos < 0 are skipped).
int draft_ingest(Ctx* c, const __nv_bfloat16* taps, const int* pos, int M, const int* row_seq, cudaStream_t s) {
  const dfl_draft_desc& d = c->d;
  const int H = d.hidden, hd = d.head_dim, Hkv = d.n_kv_heads;
  const int ntaps = d.n_taps;
  const int per = 2 * Hkv * hd, nkv = d.n_layers * per;
  if (chain_ok(c, M)) {
    std::vector<dfl_gemm_op> ops;
    ops.push_back(gop(taps, (int64_t)ntaps * H, d.fc, M, H, ntaps * H, DFL_EPI_STORE, nullptr, 0, c->dfc, H, nullptr,
                      0, nullptr, nullptr, nullptr, c->dss_ctx, d.eps));
    ops.push_back(gop(c->dfc, H, d.w_ctx_kv, M, nkv, H, DFL_EPI_STORE, nullptr, 0, c->dkvp, nkv, nullptr, 0, nullptr,
                      d.hidden_norm, c->dss_ctx, nullptr, d.eps));
    TRY(run_chain(c, ops, s));
  } else {
    TRY(gemm(c, taps, (int64_t)ntaps * H, d.fc, M, H, ntaps * H, DFL_EPI_STORE, nullptr, 0, c->dfc, H, nullptr, 0,
             nullptr, nullptr, nullptr, c->dss_ctx, d.eps, s));
    if (fused_qkv_rope(c, hd, hd) && d.n_layers <= 16) {
      // hidden_norm, every layer's k/v projection and k_norm + RoPE + append: one call
      std::vector<const void*> kn(d.n_layers);
      for (int l = 0; l < d.n_layers; ++l) kn[l] = c->dl[l].k_norm;
      return dfl_gemm_kv_append_layers(c->dfc, H, d.w_ctx_kv, M, H, d.hidden_norm, c->dss_ctx, H / 32, d.eps, c->dkvp,
                                       nkv, pos, row_seq, kn.data(), c->d_inv_freq, c->dk, c->dv,
                                       (int64_t)kv_layer_elems(c, Hkv, hd), (int64_t)Hkv * c->cap * hd,
                                       (int64_t)c->cap * hd, nullptr, 0, 0, d.n_layers, Hkv, hd, c->gemm_ws,
                                       c->gemm_ws_bytes, s);
    }
    TRY(gemm(c, c->dfc, H, d.w_ctx_kv, M, nkv, H, DFL_EPI_STORE, nullptr, 0, c->dkvp, nkv, nullptr, 0, nullptr,
             d.hidden_norm, c->dss_ctx, nullptr, d.eps, s));
  }
  for (int l = 0; l < d.n_layers; ++l) {
    __nv_bfloat16* kc = c->dk + (size_t)l * kv_layer_elems(c, Hkv, hd);
    __nv_bfloat16* vc = c->dv + (size_t)l * kv_layer_elems(c, Hkv, hd);
    TRY(dfl_qkv_rope_append(c->dkvp + (size_t)l * per, nkv, hd, pos, row_seq, c->dl[l].q_norm, c->dl[l].k_norm,
                            c->d_inv_freq, nullptr, kc, vc, (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, M, 0,
                            Hkv, hd, hd, d.eps, 0, s));
  }
  return DFL_OK;
}

// Draft block forward (DraftModel.forward_block) + lm_head argmax of every row.
int draft_block(Ctx* c, cudaStream_t s) {
  const dfl_draft_desc& d = c->d;
  const int H = d.hidden, hd = d.head_dim, Hq = d.n_heads, Hkv = d.n_kv_heads;
  const int M = c->B * c->bs;
  const int nqkv = (Hq + 2 * Hkv) * hd;
  const float eps = d.eps;
  const int* rs = c->B > 1 ? c->row_seq : nullptr;
  TRY(dfl_embed_bf16(c->block, c->t.embed, c->dh, H, M, H, c->t.vocab, c->dss, s));
  if (chain_ok(c, M)) {
    std::vector<dfl_gemm_op> ops;
    if (d.n_layers > 0)
      ops.push_back(gop(c->dh, H, c->dl[0].w_qkv, M, nqkv, H, DFL_EPI_STORE, nullptr, 0, c->dqkv, nqkv, nullptr, 0,
                        nullptr, c->dl[0].in_norm, c->dss, nullptr, eps));
    for (int l = 0; l < d.n_layers; ++l) {
      const dfl_layer_weights& w = c->dl[l];
      TRY(run_chain(c, ops, s));
      __nv_bfloat16* kc = c->dk + (size_t)l * kv_layer_elems(c, Hkv, hd);
      __nv_bfloat16* vc = c->dv + (size_t)l * kv_layer_elems(c, Hkv, hd);
      TRY(dfl_qkv_rope_append(c->dqkv, nqkv, hd, c->dpos_blk, rs, w.q_norm, w.k_norm, c->d_inv_freq, c->dq, kc, vc,
                              (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, M, Hq, Hkv, hd, hd, eps, 1, s));
      TRY(dfl_attention(c->dq, kc, vc, (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, c->dpos_blk, rs,
                        c->dkv_len, c->bs, M, Hq, Hkv, hd, d.causal, (float)(1.0 / std::sqrt((double)hd)), c->cap,
                        c->key_chunk, c->dattn, Hq * hd, nullptr, 0, 0, c->attn_ws, c->attn_ws_bytes, s));
      ops.push_back(gop(c->dattn, Hq * hd, w.w_o, M, H, Hq * hd, DFL_EPI_RESIDUAL, c->dh, H, c->dh, H, nullptr, 0,
                        nullptr, nullptr, nullptr, c->dss, eps));
      ops.push_back(gop(c->dh, H, w.w_gu, M, 2 * d.ffn, H, DFL_EPI_SILU_MUL, nullptr, 0, c->dact, d.ffn, nullptr, 0,
                        nullptr, w.post_norm, c->dss, nullptr, eps));
      ops.push_back(gop(c->dact, d.ffn, w.w_down, M, H, d.ffn, DFL_EPI_RESIDUAL, c->dh, H, c->dh, H, nullptr, 0,
                        nullptr, nullptr, nullptr, c->dss, eps));
      if (l + 1 < d.n_layers)
        ops.push_back(gop(c->dh, H, c->dl[l + 1].w_qkv, M, nqkv, H, DFL_EPI_STORE, nullptr, 0, c->dqkv, nqkv, nullptr,
                          0, nullptr, c->dl[l + 1].in_norm, c->dss, nullptr, eps));
    }
    ops.push_back(gop(c->dh, H, c->t.lm_head, M, c->t.vocab, H, DFL_EPI_ARGMAX, nullptr, 0, nullptr, 0, nullptr, 0,
                      c->dargmax, d.final_norm, c->dss, nullptr, eps));
    return run_chain(c, ops, s);
  }
  for (int l = 0; l < d.n_layers; ++l) {
    const dfl_layer_weights& w = c->dl[l];
    __nv_bfloat16* kc = c->dk + (size_t)l * kv_layer_elems(c, Hkv, hd);
    __nv_bfloat16* vc = c->dv + (size_t)l * kv_layer_elems(c, Hkv, hd);
    TRY(qkv_rope(c, c->dh, c->dss, H, w, M, Hq, Hkv, hd, hd, eps, c->dpos_blk, rs, c->d_inv_freq, c->dqkv, c->dq, kc,
                 vc, s));
    TRY(dfl_attention(c->dq, kc, vc, (int64_t)Hkv * c->cap * hd, (int64_t)c->cap * hd, c->dpos_blk, rs, c->dkv_len,
                      c->bs, M, Hq, Hkv, hd, d.causal, (float)(1.0 / std::sqrt((double)hd)), c->cap, c->key_chunk, c->dattn,
                      Hq * hd, nullptr, 0, 0, c->attn_ws, c->attn_ws_bytes, s));
    TRY(gemm(c, c->dattn, Hq * hd, w.w_o, M, H, Hq * hd, DFL_EPI_RESIDUAL, c->dh, H, c->dh, H, nullptr, 0, nullptr,
             nullptr, nullptr, c->dss, eps, s));
    TRY(gemm(c, c->dh, H, w.w_gu, M, 2 * d.ffn, H, DFL_EPI_SILU_MUL, nullptr, 0, c->dact, d.ffn, nullptr, 0,
             nullptr, w.post_norm, c->dss, nullptr, eps, s));
    TRY(gemm(c, c->dact, d.ffn, w.w_down, M, H, d.ffn, DFL_EPI_RESIDUAL, c->dh, H, c->dh, H, nullptr, 0, nullptr,
             nullptr, nullptr, c->dss, eps, s));
  }
  return gemm(c, c->dh, H, c->t.lm_head, M, c->t.vocab, H, DFL_EPI_ARGMAX, nullptr, 0, nullptr, 0, nullptr, 0,
              c->dargmax, d.final_norm, c->dss, nullptr, eps, s);
}

int draft_half(Ctx* c, cudaStream_t s) {
  const int mask = c->has_draft ? c->d.mask_token_id : 0;
  TRY(dfl_step_prepare(c->state, c->out_tokens, c->cap, c->block, c->bs, mask, c->tpos,
                       c->has_draft ? c->dpos_ctx : nullptr, c->has_draft ? c->dpos_blk : nullptr,
                       c->has_draft ? c->dkv_len : nullptr, c->B, s));
  if (!c->has_draft) return DFL_OK;
  TRY(draft_ingest(c, c->taps, c->dpos_ctx, c->B * c->bs, c->B > 1 ? c->row_seq : nullptr, s));
  TRY(draft_block(c, s));
  return dfl_draft_commit(c->state, c->dargmax, dfl_gemm_argmax_tiles(c->t.vocab), c->block, c->bs, c->inj_tok,
                          c->inj_tok_stride, c->inj_len, c->inj_len_stride, c->inj_noise, c->inj_noise_stride, c->B,
                          s);
}

int verify_half(Ctx* c, cudaStream_t s) {
  TRY(target_forward(c, c->block, c->tpos, c->B * c->bs, c->B > 1 ? c->row_seq : nullptr, c->bs, c->cap, c->taps,
                     s));
  return dfl_verify_accept(c->state, c->argmax, dfl_gemm_argmax_tiles(c->t.vocab), c->block, c->bs, c->out_tokens,
                           c->cap, nullptr, c->stop_ids, c->n_stop, c->accept_log, c->max_steps, c->B, s);
}

// Records fn on the private stream into an executable graph.
int capture(Ctx* c, int (*fn)(Ctx*, cudaStream_t), cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return fail_cuda("capture: begin", e);
  const int st = fn(c, c->cap_stream);
  e = cudaStreamEndCapture(c->cap_stream, &g);
  if (st != DFL_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  if (e != cudaSuccess) return fail_cuda("capture: end", e);
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail_cuda("capture: instantiate", e);
  return DFL_OK;
}

int run_half(Ctx* c, int (*fn)(Ctx*, cudaStream_t), cudaGraphExec_t* g, void* stream) {
  cudaStream_t s = dfl::as_stream(stream);
  if (!c->use_graph) return fn(c, s);
  if (!*g) {
    // the private stream waits for the caller's work so far; captured work is recorded, not run
    TRY(capture(c, fn, g));
  }
  cudaError_t e = cudaGraphLaunch(*g, s);
  return e == cudaSuccess ? DFL_OK : fail_cuda("cudaGraphLaunch", e);
}

void release(Ctx* c) {
  if (c->g_draft) cudaGraphExecDestroy(c->g_draft);
  if (c->g_verify) cudaGraphExecDestroy(c->g_verify);
  if (c->cap_stream) cudaStreamDestroy(c->cap_stream);
  for (auto& b : c->owned) cudaFree(b.p);
  delete c;
}

void inv_freq_host(std::vector<float>& out, int rot_dim, float theta) {
  out.resize(rot_dim / 2);
  for (int i = 0; i < rot_dim / 2; ++i) out[i] = (float)(1.0 / std::pow((double)theta, (2.0 * i) / rot_dim));
}

}  // namespace

extern "C" int dfl_ctx_create(const dfl_qwen3_desc* target, const dfl_draft_desc* draft, int batch, int max_total,
                              int block_size, const int32_t* stop_ids, int n_stop, int max_steps, int flags,
                              dfl_ctx** out) {
  if (!target || !out || batch <= 0 || max_total <= 0 || block_size <= 0 || n_stop < 0 || (n_stop && !stop_ids)) {
    set_error("dfl_ctx_create: invalid arguments");
    return DFL_ERR_INVALID;
  }
  *out = nullptr;
  if (!target->embed || !target->lm_head || !target->final_norm || !target->layers || target->n_layers < 0 ||
      target->hidden % 256 || target->head_dim <= 0 || target->n_kv_heads <= 0 ||
      target->n_heads % target->n_kv_heads) {
    set_error("dfl_ctx_create: incomplete or unsupported target description");
    return DFL_ERR_INVALID;
  }
  if (block_size > 1 && !draft) {
    set_error("dfl_ctx_create: a block size above 1 needs a draft");
    return DFL_ERR_INVALID;
  }
  if (draft && (draft->block_size < block_size || draft->n_taps <= 0 || !draft->target_layer_ids || !draft->fc ||
                !draft->w_ctx_kv || !draft->layers || draft->hidden != target->hidden)) {
    set_error("dfl_ctx_create: incomplete or inconsistent draft description");
    return DFL_ERR_INVALID;
  }
  Ctx* c = new Ctx();
  c->t = *target;
  c->tl.assign(target->layers, target->layers + target->n_layers);
  c->has_draft = draft != nullptr && block_size > 1;
  if (c->has_draft) {
    c->d = *draft;
    c->dl.assign(draft->layers, draft->layers + draft->n_layers);
    c->tap_ids.assign(draft->target_layer_ids, draft->target_layer_ids + draft->n_taps);
    for (size_t i = 1; i < c->tap_ids.size(); ++i)
      if (c->tap_ids[i] <= c->tap_ids[i - 1]) {
        set_error("dfl_ctx_create: target_layer_ids must be strictly ascending");
        release(c);
        return DFL_ERR_INVALID;
      }
  }
  c->B = batch;
  c->bs = block_size;
  c->cap = max_total + 2 * block_size + 1;
  c->max_steps = max_steps > 0 ? max_steps : max_total + 1;
  c->batched = batch >= 4;
  c->key_chunk = c->batched ? 1024 : 64;  // as the Python host's SpecSession
  c->wide_split_max = c->batched ? (batch < 16 ? 4 : 1) : 1;
  c->use_graph = !(flags & DFL_CTX_NO_GRAPH);
  {
    const char* e = getenv("DFLASH_B200_GEMM_CHAIN");  // opt-in, as the Python host
    c->use_chain = e && e[0] == '1';
  }
  c->n_stop = n_stop;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&c->n_sm, cudaDevAttrMultiProcessorCount, dev);
  const int M = batch * block_size;
  const int PREFILL = 128;
  c->max_rows = M > PREFILL ? M : PREFILL;
  const dfl_qwen3_desc& t = c->t;
  const int H = t.hidden, ntaps = c->has_draft ? c->d.n_taps : 1;
  int st = DFL_OK;
#define A(ptr, n)                              \
  if ((st = alloc(c, &(ptr), (n))) != DFL_OK) { \
    release(c);                                \
    return st;                                 \
  }
  A(c->state, (size_t)batch);
  A(c->out_tokens, (size_t)batch * c->cap);
  A(c->block, (size_t)M);
  A(c->tpos, (size_t)M);
  A(c->dpos_ctx, (size_t)M);
  A(c->dpos_blk, (size_t)M);
  A(c->dkv_len, (size_t)batch);
  A(c->row_seq, (size_t)c->max_rows);
  A(c->accept_log, (size_t)batch * c->max_steps);
  A(c->stop_ids, (size_t)(n_stop > 0 ? n_stop : 1));
  A(c->prefill_tok, (size_t)PREFILL);
  A(c->prefill_pos, (size_t)PREFILL);
  A(c->first_tok, (size_t)1);
  A(c->tk, (size_t)t.n_layers * kv_layer_elems(c, t.n_kv_heads, t.head_dim));
  A(c->tv, (size_t)t.n_layers * kv_layer_elems(c, t.n_kv_heads, t.head_dim));
  A(c->taps, (size_t)c->max_rows * ntaps * H);
  const int R = c->max_rows;
  A(c->h, (size_t)R * H);
  A(c->qkv, (size_t)R * (t.n_heads + 2 * t.n_kv_heads) * t.head_dim);
  A(c->q, (size_t)R * t.n_heads * t.head_dim);
  A(c->attn, (size_t)R * t.n_heads * t.head_dim);
  A(c->act, (size_t)R * t.ffn);
  A(c->ss, (size_t)R * (H / 32));
  const int vt = dfl_gemm_argmax_tiles(t.vocab);
  A(c->argmax, (size_t)R * vt * 2);
  std::vector<float> f;
  inv_freq_host(f, t.rope_dim, t.rope_theta);
  A(c->t_inv_freq, f.size());
  cudaMemcpy(c->t_inv_freq, f.data(), f.size() * sizeof(float), cudaMemcpyHostToDevice);
  // (N, K) of every weight, for the scratch sizes
  std::vector<std::pair<int, int>> nk = {{(t.n_heads + 2 * t.n_kv_heads) * t.head_dim, H},
                                         {H, t.n_heads * t.head_dim},
                                         {2 * t.ffn, H},
                                         {H, t.ffn},
                                         {t.vocab, H}};
  std::vector<std::pair<int, int>> heads = {{t.n_heads, t.head_dim}};
  if (c->has_draft) {
    const dfl_draft_desc& d = c->d;
    A(c->dk, (size_t)d.n_layers * kv_layer_elems(c, d.n_kv_heads, d.head_dim));
    A(c->dv, (size_t)d.n_layers * kv_layer_elems(c, d.n_kv_heads, d.head_dim));
    A(c->dh, (size_t)M * H);
    A(c->dqkv, (size_t)M * (d.n_heads + 2 * d.n_kv_heads) * d.head_dim);
    A(c->dq, (size_t)M * d.n_heads * d.head_dim);
    A(c->dattn, (size_t)M * d.n_heads * d.head_dim);
    A(c->dact, (size_t)M * d.ffn);
    A(c->dss, (size_t)M * (H / 32));
    A(c->dargmax, (size_t)M * vt * 2);
    A(c->dfc, (size_t)R * H);
    A(c->dss_ctx, (size_t)R * (H / 32));
    A(c->dkvp, (size_t)R * d.n_layers * 2 * d.n_kv_heads * d.head_dim);
    inv_freq_host(f, d.head_dim, d.rope_theta);
    A(c->d_inv_freq, f.size());
    cudaMemcpy(c->d_inv_freq, f.data(), f.size() * sizeof(float), cudaMemcpyHostToDevice);
    nk.push_back({H, d.n_taps * H});
    nk.push_back({d.n_layers * 2 * d.n_kv_heads * d.head_dim, H});
    nk.push_back({(d.n_heads + 2 * d.n_kv_heads) * d.head_dim, H});
    nk.push_back({H, d.n_heads * d.head_dim});
    nk.push_back({2 * d.ffn, H});
    nk.push_back({H, d.ffn});
    heads.push_back({d.n_heads, d.head_dim});
  }
  if (n_stop > 0) cudaMemcpy(c->stop_ids, stop_ids, sizeof(int) * n_stop, cudaMemcpyHostToDevice);
  // row -> sequence map of a step block
  {
    std::vector<int> rs(c->max_rows, 0);
    for (int r = 0; r < M; ++r) rs[r] = r / block_size;
    cudaMemcpy(c->row_seq, rs.data(), sizeof(int) * M, cudaMemcpyHostToDevice);
  }
  size_t gneed = 0, wneed = 0, aneed = 0;
  for (int rows : {M, PREFILL}) {
    for (auto& p : nk) {
      gneed = std::max(gneed, dfl_gemm_workspace_bytes(rows, p.first, p.second, 0));
      wneed = std::max(wneed, dfl_gemm_wide_workspace_bytes(rows, p.first, p.second, 1, wide_split(c, p.first,
                                                                                                  p.second)));
    }
    for (auto& hh : heads)
      aneed = std::max(aneed, dfl_attention_workspace_bytes(rows, hh.first, hh.second, c->cap, c->key_chunk));
  }
  unsigned char *gw = nullptr, *ww = nullptr, *aw = nullptr, *cw = nullptr;
  const size_t chain_bytes = 6u << 20;  // as the Python host's Workspace.CHAIN_BYTES (counters + partials)
  A(cw, chain_bytes);  // zero-filled: the chain's counters start at zero
  c->chain_ws = cw;
  c->chain_ws_bytes = chain_bytes;
  A(gw, gneed);  // zero-filled: the split-K counters start at zero
  A(aw, aneed);
  c->gemm_ws = gw;
  c->gemm_ws_bytes = gneed;
  c->attn_ws = aw;
  c->attn_ws_bytes = aneed;
  if (c->batched) {
    A(ww, wneed);
    c->wide_ws = ww;
    c->wide_ws_bytes = wneed;
  }
#undef A
  cudaError_t e = cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    release(c);
    return fail_cuda("dfl_ctx_create", e);
  }
  *out = reinterpret_cast<dfl_ctx*>(c);
  return DFL_OK;
}

extern "C" int dfl_ctx_destroy(dfl_ctx* ctx) {
  if (!ctx) return DFL_OK;
  cudaDeviceSynchronize();
  release(reinterpret_cast<Ctx*>(ctx));
  return DFL_OK;
}

extern "C" int dfl_ctx_prefill(dfl_ctx* ctx, int seq, const int32_t* tokens, int n_tokens, int max_new_tokens,
                               void* stream) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c || !tokens || seq < 0 || seq >= c->B || n_tokens <= 0 || max_new_tokens < 0) {
    set_error("dfl_ctx_prefill: invalid arguments");
    return DFL_ERR_INVALID;
  }
  if (n_tokens + max_new_tokens + 2 * c->bs + 1 > c->cap) {
    set_error("dfl_ctx_prefill: prompt + max_new_tokens exceeds the context capacity");
    return DFL_ERR_INVALID;
  }
  cudaStream_t s = dfl::as_stream(stream);
  const int CH = 128;
  const int ntaps = (int)c->tap_ids.size();
  std::vector<int> pos(CH), seqmap(CH, seq);
  cudaError_t e = cudaSuccess;
  // batched contexts: the prefill rows all belong to `seq`; the row map is overwritten
  // for the prefill and restored afterwards
  const int* prs = c->B > 1 ? c->row_seq : nullptr;
  for (int c0 = 0; c0 < n_tokens; c0 += CH) {
    const int n = std::min(CH, n_tokens - c0);
    for (int i = 0; i < n; ++i) pos[i] = c0 + i;
    // synchronous copies: the prefill is a set-up call (the step calls never sync)
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return fail_cuda("dfl_ctx_prefill", e);
    cudaMemcpy(c->prefill_tok, tokens + c0, sizeof(int) * n, cudaMemcpyHostToDevice);
    cudaMemcpy(c->prefill_pos, pos.data(), sizeof(int) * n, cudaMemcpyHostToDevice);
    if (prs) cudaMemcpy(c->row_seq, seqmap.data(), sizeof(int) * n, cudaMemcpyHostToDevice);
    TRY(target_forward(c, c->prefill_tok, c->prefill_pos, n, prs, n, c0 + n, ntaps ? c->taps : nullptr, s));
    if (c->has_draft) TRY(draft_ingest(c, c->taps, c->prefill_pos, n, prs, s));
    if (c0 + n == n_tokens)
      TRY(dfl_argmax_reduce(c->argmax + (size_t)(n - 1) * dfl_gemm_argmax_tiles(c->t.vocab) * 2, 1,
                            dfl_gemm_argmax_tiles(c->t.vocab), c->first_tok, s));
  }
  if (c->B > 1) {  // restore the step block's row map
    std::vector<int> m(c->B * c->bs);
    for (int r = 0; r < c->B * c->bs; ++r) m[r] = r / c->bs;
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return fail_cuda("dfl_ctx_prefill", e);
    cudaMemcpy(c->row_seq, m.data(), sizeof(int) * m.size(), cudaMemcpyHostToDevice);
  }
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return fail_cuda("dfl_ctx_prefill", e);
  int first = 0;
  cudaMemcpy(&first, c->first_tok, sizeof(int), cudaMemcpyDeviceToHost);
  std::vector<int> stops(c->n_stop);
  if (c->n_stop) cudaMemcpy(stops.data(), c->stop_ids, sizeof(int) * c->n_stop, cudaMemcpyDeviceToHost);
  int* row = c->out_tokens + (size_t)seq * c->cap;
  cudaMemcpy(row, tokens, sizeof(int) * n_tokens, cudaMemcpyHostToDevice);
  cudaMemcpy(row + n_tokens, &first, sizeof(int), cudaMemcpyHostToDevice);
  dfl_seq_state st;
  std::memset(&st, 0, sizeof(st));
  const int total = n_tokens + max_new_tokens;
  st.start = n_tokens;
  st.pending = 0;
  st.draft_len = n_tokens;
  st.finished = n_tokens + 1 > total;
  st.stop_index = -1;
  for (int x : stops)
    if (x == first) st.stop_index = n_tokens;
  st.total_max = total;
  st.prompt_len = n_tokens;
  cudaMemcpy(c->state + seq, &st, sizeof(st), cudaMemcpyHostToDevice);
  cudaMemset(c->accept_log + (size_t)seq * c->max_steps, 0, sizeof(int) * c->max_steps);
  e = cudaDeviceSynchronize();
  return e == cudaSuccess ? DFL_OK : fail_cuda("dfl_ctx_prefill", e);
}

extern "C" int dfl_ctx_set_injection(dfl_ctx* ctx, const int32_t* trace, int64_t trace_stride, const int32_t* lengths,
                                     int64_t lengths_stride, const int32_t* noise, int64_t noise_stride) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c || (trace && (!lengths || !noise))) {
    set_error("dfl_ctx_set_injection: invalid arguments");
    return DFL_ERR_INVALID;
  }
  c->inj_tok = trace;
  c->inj_len = lengths;
  c->inj_noise = noise;
  c->inj_tok_stride = trace_stride;
  c->inj_len_stride = lengths_stride;
  c->inj_noise_stride = noise_stride;
  if (c->g_draft) {  // the recorded draft half holds the old pointers
    cudaGraphExecDestroy(c->g_draft);
    c->g_draft = nullptr;
  }
  return DFL_OK;
}

extern "C" int dfl_draft_step(dfl_ctx* ctx, void* stream) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c) {
    set_error("dfl_draft_step: null context");
    return DFL_ERR_INVALID;
  }
  return run_half(c, draft_half, &c->g_draft, stream);
}

extern "C" int dfl_verify_step(dfl_ctx* ctx, void* stream) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c) {
    set_error("dfl_verify_step: null context");
    return DFL_ERR_INVALID;
  }
  return run_half(c, verify_half, &c->g_verify, stream);
}

extern "C" int dfl_rollback(dfl_ctx* ctx, void* stream) {
  (void)stream;
  if (!ctx) {
    set_error("dfl_rollback: null context");
    return DFL_ERR_INVALID;
  }
  // dense targets: dfl_verify_step's accept already moved every sequence's cache length
  // to start + accepted (the next block overwrites the rejected slots)
  return DFL_OK;
}

extern "C" int dfl_ctx_buffers(dfl_ctx* ctx, dfl_seq_state** state, int32_t** out_tokens, int64_t* out_stride,
                               int32_t** accept_log, int64_t* log_stride) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c) {
    set_error("dfl_ctx_buffers: null context");
    return DFL_ERR_INVALID;
  }
  if (state) *state = c->state;
  if (out_tokens) *out_tokens = c->out_tokens;
  if (out_stride) *out_stride = c->cap;
  if (accept_log) *accept_log = c->accept_log;
  if (log_stride) *log_stride = c->max_steps;
  return DFL_OK;
}

extern "C" int dfl_ctx_read(dfl_ctx* ctx, dfl_seq_state* state, int32_t* out_tokens, void* stream) {
  Ctx* c = reinterpret_cast<Ctx*>(ctx);
  if (!c) {
    set_error("dfl_ctx_read: null context");
    return DFL_ERR_INVALID;
  }
  cudaStream_t s = dfl::as_stream(stream);
  cudaError_t e = cudaSuccess;
  if (state) e = cudaMemcpyAsync(state, c->state, sizeof(dfl_seq_state) * c->B, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && out_tokens)
    e = cudaMemcpyAsync(out_tokens, c->out_tokens, sizeof(int) * (size_t)c->B * c->cap, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? DFL_OK : fail_cuda("dfl_ctx_read", e);
}
