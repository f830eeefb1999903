// Row-wise layer kernels of the Qwen3 / DFlash decoder layers.
//
//  * dfl_rmsnorm_bf16     - nn.RMSNorm / mx.fast.rms_norm (input_layernorm,
//                           post_attention_layernorm, final norm, the draft's
//                           hidden_norm: draft.py:167-171, 198-201)
//  * dfl_embed_bf16       - nn.Embedding row gather (adapters.py:603-604, runtime.py:410)
//  * dfl_qkv_rope_append  - per-head q_norm/k_norm, non-interleaved RoPE and the
//                           KV-cache append of mlx-lm KVCache.update_and_fetch
//                           (draft.py:123-147; mlx-lm qwen3 Attention)
//
// All kernels are one warp per row (or per row x head): the reduction order of a
// row never depends on how many rows a launch carries.
#include "common.cuh"
#include "rope.cuh"

namespace dfl {

// -------------------------------------------------------------------------
// RMSNorm: y = w * (x * rsqrt(mean(x^2) + eps)), fp32 math, one rounding.
// -------------------------------------------------------------------------
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
                               __nv_bfloat16* __restrict__ y, long long ldy, int M, int H, float eps) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= M) return;
  const __nv_bfloat16* xr = x + (long long)row * ldx;
  __nv_bfloat16* yr = y + (long long)row * ldy;
  // H % 256 == 0 path: each lane owns 8-element vectors at stride 256
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = bf2f(e[j]);
      ss += f * f;
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)H + eps);
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    uint4 wv = w ? *reinterpret_cast<const uint4*>(w + c) : make_uint4(0, 0, 0, 0);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint4 o;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float wf = w ? bf2f(we[j]) : 1.f;
      oe[j] = f2bf(wf * (bf2f(e[j]) * inv));
    }
    *reinterpret_cast<uint4*>(yr + c) = o;
  }
}

// -------------------------------------------------------------------------
// Embedding gather: y[r] = table[tok[r]]  (tok < 0 or >= V gives zeros)
// -------------------------------------------------------------------------
__global__ void embed_kernel(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ y, long long ldy, int M, int H, int V,
                             float* __restrict__ sumsq) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int row = blockIdx.x;
  if (row >= M) return;
  const int t = tok[row];
  __nv_bfloat16* yr = y + (long long)row * ldy;
  // blockDim.x is a multiple of 4: four lanes cover one 32-column group
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t >= 0 && t < V) v = *reinterpret_cast<const uint4*>(table + (long long)t * H + c);
    *reinterpret_cast<uint4*>(yr + c) = v;
    if (sumsq) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += bf2f(e[k]) * bf2f(e[k]);
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      if ((threadIdx.x & 3) == 0) sumsq[(long long)row * (H / 32) + c / 32] = ss;
    }
  }
}

__global__ void qkv_rope_append_kernel(QkvArgs a) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  extern __shared__ float sh[];  // [warps][hd]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nheads = a.Hq + 2 * a.Hkv;
  const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (item >= (long long)a.M * nheads) return;
  qkv_rope_row(a, (int)(item / nheads), (int)(item % nheads), lane, sh + warp * a.hd);
}

}  // namespace dfl

using namespace dfl;

extern "C" int dfl_rmsnorm_bf16(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, int M, int H,
                                float eps, void* stream) {
  if (M == 0) return DFL_OK;
  if (!x || !y || M < 0 || H <= 0) {
    set_error("dfl_rmsnorm_bf16: bad arguments");
    return DFL_ERR_INVALID;
  }
  if (H % 256 || ldx % 8 || ldy % 8) {
    set_error("dfl_rmsnorm_bf16: H must be a multiple of 256 and rows 16-byte aligned (H=%d)", H);
    return DFL_ERR_UNSUPPORTED;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((M + 3) / 4);
  cfg.blockDim = dim3(128);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, rmsnorm_kernel, static_cast<const __nv_bfloat16*>(x), (long long)ldx,
                                     static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y),
                                     (long long)ldy, M, H, eps);
  if (e != cudaSuccess) {
    set_error("dfl_rmsnorm_bf16: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_embed_bf16(const int32_t* tokens, const void* table, void* y, int64_t ldy, int M, int H, int V,
                              float* sumsq_out, void* stream) {
  if (M == 0) return DFL_OK;
  if (!tokens || !table || !y || H % 8 || ldy % 8 || (sumsq_out && H % 256)) {
    set_error("dfl_embed_bf16: bad arguments (H %% 8 == 0; H %% 256 == 0 with sumsq_out)");
    return DFL_ERR_INVALID;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(128);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, embed_kernel, tokens, static_cast<const __nv_bfloat16*>(table),
                                     static_cast<__nv_bfloat16*>(y), (long long)ldy, M, H, V, sumsq_out);
  if (e != cudaSuccess) {
    set_error("dfl_embed_bf16: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

static int qkv_rope_append_impl(const void* qkv, int64_t ldqkv, int q_stride, const int32_t* pos,
                                   const int32_t* row_seq, const void* q_norm, const void* k_norm,
                                   const float* inv_freq, void* q_out, void* k_cache, void* v_cache,
                                   int64_t seq_stride, int64_t head_stride, int M, int Hq, int Hkv, int hd,
                                   int rot_dim, float eps, int do_q, void* stream, const int32_t* page_table, int64_t pt_stride, int page_size) {
  if (M == 0) return DFL_OK;
  if (!qkv || !pos || !q_norm || !k_norm || !inv_freq || !k_cache || !v_cache || (do_q && !q_out)) {
    set_error("dfl_qkv_rope_append: null pointer");
    return DFL_ERR_INVALID;
  }
  if (hd <= 0 || hd > 512 || rot_dim < 0 || rot_dim > hd || (rot_dim & 1) || Hq < 0 || Hkv <= 0) {
    set_error("dfl_qkv_rope_append: bad head geometry hd=%d rot_dim=%d", hd, rot_dim);
    return DFL_ERR_INVALID;
  }
  QkvArgs a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ldqkv = ldqkv;
  a.q_stride = q_stride;
  a.pos = pos;
  a.row_seq = row_seq;
  a.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  a.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  a.inv_freq = inv_freq;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.seq_stride = seq_stride;
  a.head_stride = head_stride;
  a.M = M;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.hd = hd;
  a.rot_dim = rot_dim;
  a.eps = eps;
  a.do_q = do_q;
  a.page_table = page_table;
  a.pt_stride = pt_stride;
  a.page_shift = 0;
  a.layer_stride = 0;
  if (page_table) {
    if (page_size < 64 || (page_size & (page_size - 1)) || pt_stride <= 0) {
      set_error("dfl_qkv_rope_append_paged: page_size must be a power of two >= 64 (got %d)", page_size);
      return DFL_ERR_INVALID;
    }
    while ((1 << a.page_shift) < page_size) ++a.page_shift;
  }
  const long long items = (long long)M * (Hq + 2 * Hkv);
  const int warps = 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((items + warps - 1) / warps));
  cfg.blockDim = dim3(32 * warps);
  cfg.dynamicSmemBytes = warps * hd * sizeof(float);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qkv_rope_append_kernel, a);
  if (e != cudaSuccess) {
    set_error("dfl_qkv_rope_append: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_qkv_rope_append(const void* qkv, int64_t ldqkv, int q_stride, const int32_t* pos,
                                   const int32_t* row_seq, const void* q_norm, const void* k_norm,
                                   const float* inv_freq, void* q_out, void* k_cache, void* v_cache,
                                   int64_t seq_stride, int64_t head_stride, int M, int Hq, int Hkv, int hd,
                                   int rot_dim, float eps, int do_q, void* stream) {
  return qkv_rope_append_impl(qkv, ldqkv, q_stride, pos, row_seq, q_norm, k_norm, inv_freq, q_out, k_cache, v_cache,
                              seq_stride, head_stride, M, Hq, Hkv, hd, rot_dim, eps, do_q, stream, nullptr, 0, 0);
}

extern "C" int dfl_qkv_rope_append_paged(const void* qkv, int64_t ldqkv, int q_stride, const int32_t* pos,
                                         const int32_t* row_seq, const void* q_norm, const void* k_norm,
                                         const float* inv_freq, void* q_out, void* k_pages, void* v_pages,
                                         int64_t page_stride, int64_t head_stride, const int32_t* page_table,
                                         int64_t pt_stride, int page_size, int M, int Hq, int Hkv, int hd, int rot_dim,
                                         float eps, int do_q, void* stream) {
  if (!page_table) {
    set_error("dfl_qkv_rope_append_paged: null page table");
    return DFL_ERR_INVALID;
  }
  return qkv_rope_append_impl(qkv, ldqkv, q_stride, pos, row_seq, q_norm, k_norm, inv_freq, q_out, k_pages, v_pages,
                              page_stride, head_stride, M, Hq, Hkv, hd, rot_dim, eps, do_q, stream, page_table,
                              pt_stride, page_size);
}
