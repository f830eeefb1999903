// Gated-delta-net (Qwen3.5 linear-attention) layer kernels around the recurrence.
//
//  * dfl_gdn_prep      depthwise causal conv1d (k = 4) + SiLU over [conv state | qkv],
//                      split into q / k / v, q <- Dk^-1 * rmsnorm(q), k <- Dk^-1/2 *
//                      rmsnorm(k), beta = sigmoid(b), g = exp(-exp(A_log) *
//                      softplus(a + dt_bias)); keeps the conv window for rollback.
//                      (custom_qwen35_model.py:409-450; mlx-lm compute_g)
//  * dfl_gdn_rollback  cache rollback to "after `accepted` tokens": recurrent state
//                      <- per-token snapshot accepted-1, conv state <- window rows
//                      [accepted, accepted + K - 1) (custom_qwen35_model.py:1029-1074,
//                      where the reference replays the recurrence instead).
//  * dfl_gated_rmsnorm RMSNormGated: rmsnorm(o) * w * silu(z) per value head
//                      (adapters.py:226-227, Qwen3-Next RMSNormGated).
//
// Row r of a launch belongs to sequence r / T (token r % T). All reductions are per
// row (warp) so results do not depend on how many rows a launch carries.
#include "common.cuh"

namespace dfl {

struct GdnPrepArgs {
  const __nv_bfloat16* proj;  // [B*T, ldp]: [qkv (C) | z (Hv*Dv) | b (Hv) | a (Hv)]
  long long ldp;
  const __nv_bfloat16* conv_w;  // [C][4]
  const float* A_log;
  const float* dt_bias;
  const __nv_bfloat16* conv_state;  // [B][3][C] state before this block
  __nv_bfloat16* window;            // [B][>= 3+T][C] (nullable), win_stride elements per sequence
  long long win_stride;
  __nv_bfloat16* q;                 // [B*T][Hk][Dk]
  __nv_bfloat16* k;
  __nv_bfloat16* v;  // [B*T][Hv][Dv]
  float* g;          // [B*T][Hv]
  float* beta;
  int B, T, Hk, Hv, Dk, Dv, C;
  float eps;
};

// one CTA per token row; threads stride over the conv channels, then one warp per
// q / k head for the norms and one thread per value head for g / beta
__global__ void gdn_prep_kernel(GdnPrepArgs a) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  extern __shared__ float sh[];  // conv output of this row [C]
  const int row = blockIdx.x;
  const int b = row / a.T, t = row % a.T;
  const __nv_bfloat16* cs = a.conv_state + (long long)b * 3 * a.C;
  const __nv_bfloat16* pr = a.proj + (long long)row * a.ldp;
  for (int c = threadIdx.x; c < a.C; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = t - 3 + j;  // index into [state (3) | block (T)] minus 3
      const float x = i < 0 ? bf2f(cs[(long long)(3 + i) * a.C + c])
                            : bf2f(a.proj[(long long)(b * a.T + i) * a.ldp + c]);
      acc += bf2f(a.conv_w[c * 4 + j]) * x;
    }
    const float cv = round_bf16(acc);
    sh[c] = round_bf16(cv / (1.f + __expf(-cv)));
    if (a.window) {
      __nv_bfloat16* w = a.window + (long long)b * a.win_stride;
      w[(long long)(3 + t) * a.C + c] = pr[c];
      if (t == 0)
        for (int j = 0; j < 3; ++j) w[(long long)j * a.C + c] = cs[(long long)j * a.C + c];
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int kd = a.Hk * a.Dk;
  // q heads then k heads: per-head rmsnorm without weight, scaled
  for (int hh = warp; hh < 2 * a.Hk; hh += nw) {
    const bool isq = hh < a.Hk;
    const int h = isq ? hh : hh - a.Hk;
    const float* src = sh + (isq ? 0 : kd) + h * a.Dk;
    float ss = 0.f;
    for (int i = lane; i < a.Dk; i += 32) ss += src[i] * src[i];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)a.Dk + a.eps);
    const float sc = isq ? 1.f / (float)a.Dk : rsqrtf((float)a.Dk);
    __nv_bfloat16* dst = (isq ? a.q : a.k) + ((long long)row * a.Hk + h) * a.Dk;
    for (int i = lane; i < a.Dk; i += 32) dst[i] = f2bf(sc * round_bf16(src[i] * inv));
  }
  for (int i = threadIdx.x; i < a.Hv * a.Dv; i += blockDim.x) a.v[(long long)row * a.Hv * a.Dv + i] = f2bf(sh[2 * kd + i]);
  for (int h = threadIdx.x; h < a.Hv; h += blockDim.x) {
    const float bb = bf2f(pr[a.C + a.Hv * a.Dv + h]);
    const float aa = bf2f(pr[a.C + a.Hv * a.Dv + a.Hv + h]);
    const float x = aa + a.dt_bias[h];
    const float sp = x > 20.f ? x : log1pf(__expf(x));
    a.g[(long long)row * a.Hv + h] = __expf(-__expf(a.A_log[h]) * sp);
    a.beta[(long long)row * a.Hv + h] = 1.f / (1.f + __expf(-bb));
  }
}

// state[b] <- snaps[b][acc-1]; conv_state[b] <- window[b][acc .. acc+2]. Every block of
// sequence b copies a 1/gridDim.x share of both with 16-byte moves (the conv rows are
// 3*C bf16, a multiple of 8 elements).
__global__ void gdn_rollback_kernel(float* __restrict__ state, const float* __restrict__ snaps,
                                    __nv_bfloat16* __restrict__ conv_state, const __nv_bfloat16* __restrict__ window,
                                    const int* __restrict__ accepted, int acc_stride, int T, long long S, int C,
                                    long long win_stride) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int b = blockIdx.y;
  const int acc = accepted[(long long)b * acc_stride];
  if (acc < 1 || acc > T) return;
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x, nthr = (long long)gridDim.x * blockDim.x;
  if (snaps) {
    const float4* src = reinterpret_cast<const float4*>(snaps + ((long long)b * T + acc - 1) * S);
    float4* dst = reinterpret_cast<float4*>(state + (long long)b * S);
    for (long long i = tid; i < S / 4; i += nthr) dst[i] = src[i];
  }
  if (window) {
    const uint4* src = reinterpret_cast<const uint4*>(window + (long long)b * win_stride + (long long)acc * C);
    uint4* dst = reinterpret_cast<uint4*>(conv_state + (long long)b * 3 * C);
    for (long long i = tid; i < 3LL * C / 8; i += nthr) dst[i] = src[i];
  }
}

// out[r, h*Dv + d] = bf16( bf16(w[d] * o * rsqrt(mean(o^2)+eps)) * bf16(silu(z)) ), one warp per (row, head)
__global__ void gated_rmsnorm_kernel(const __nv_bfloat16* __restrict__ o, long long ldo, const __nv_bfloat16* __restrict__ z,
                                     long long ldz, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                     long long ldout, int M, int H, int D, float eps) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (item >= (long long)M * H) return;
  const int r = (int)(item / H), h = (int)(item % H);
  const __nv_bfloat16* src = o + (long long)r * ldo + (long long)h * D;
  float ss = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float f = bf2f(src[i]);
    ss += f * f;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
  const __nv_bfloat16* zr = z + (long long)r * ldz + (long long)h * D;
  __nv_bfloat16* dst = out + (long long)r * ldout + (long long)h * D;
  for (int i = lane; i < D; i += 32) {
    const float xn = round_bf16(bf2f(w[i]) * (bf2f(src[i]) * inv));
    const float zz = bf2f(zr[i]);
    const float sz = round_bf16(zz / (1.f + __expf(-zz)));
    dst[i] = f2bf(xn * sz);
  }
}

static cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace dfl

using namespace dfl;

extern "C" int dfl_gdn_prep(const void* proj, int64_t ldp, const void* conv_w, const float* A_log, const float* dt_bias,
                            const void* conv_state, void* window, int64_t win_stride, void* q, void* k, void* v,
                            float* g, float* beta, int B, int T, int Hk, int Hv, int Dk, int Dv, float eps,
                            void* stream) {
  if (B == 0 || T == 0) return DFL_OK;
  if (!proj || !conv_w || !A_log || !dt_bias || !conv_state || !q || !k || !v || !g || !beta || B < 0 || T < 0 ||
      Hk <= 0 || Hv <= 0 || Dk <= 0 || Dv <= 0) {
    set_error("dfl_gdn_prep: bad arguments");
    return DFL_ERR_INVALID;
  }
  const int C = 2 * Hk * Dk + Hv * Dv;
  if ((size_t)C * sizeof(float) > 200 * 1024) {
    set_error("dfl_gdn_prep: conv width %d too large", C);
    return DFL_ERR_UNSUPPORTED;
  }
  GdnPrepArgs a;
  a.proj = static_cast<const __nv_bfloat16*>(proj);
  a.ldp = ldp;
  a.conv_w = static_cast<const __nv_bfloat16*>(conv_w);
  a.A_log = A_log;
  a.dt_bias = dt_bias;
  a.conv_state = static_cast<const __nv_bfloat16*>(conv_state);
  a.window = static_cast<__nv_bfloat16*>(window);
  a.win_stride = win_stride > 0 ? win_stride : (long long)(3 + T) * C;
  a.q = static_cast<__nv_bfloat16*>(q);
  a.k = static_cast<__nv_bfloat16*>(k);
  a.v = static_cast<__nv_bfloat16*>(v);
  a.g = g;
  a.beta = beta;
  a.B = B;
  a.T = T;
  a.Hk = Hk;
  a.Hv = Hv;
  a.Dk = Dk;
  a.Dv = Dv;
  a.C = C;
  a.eps = eps;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    init = true;
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(B * T), dim3(512), (size_t)C * sizeof(float), as_stream(stream), attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_prep_kernel, a);
  if (e != cudaSuccess) {
    set_error("dfl_gdn_prep: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_gdn_rollback(float* state, const float* snapshots, void* conv_state, const void* window,
                                int64_t win_stride, const int32_t* accepted, int acc_stride, int B, int T, int Hv,
                                int Dv, int Dk, int C, void* stream) {
  if (B == 0) return DFL_OK;
  if (!accepted || (snapshots && !state) || (window && !conv_state) || T <= 0 || B < 0) {
    set_error("dfl_gdn_rollback: bad arguments");
    return DFL_ERR_INVALID;
  }
  const long long S = (long long)Hv * Dv * Dk;
  const long long ws = win_stride > 0 ? win_stride : (long long)(3 + T) * C;
  if (S % 4 || C % 8 || ws % 8 || (reinterpret_cast<uintptr_t>(window) | reinterpret_cast<uintptr_t>(conv_state)) & 15) {
    set_error("dfl_gdn_rollback: state size %% 4, channels %% 8 and 16-byte aligned conv buffers needed");
    return DFL_ERR_UNSUPPORTED;
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(64, B), dim3(256), 0, as_stream(stream), attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_rollback_kernel, state, snapshots,
                                     static_cast<__nv_bfloat16*>(conv_state),
                                     static_cast<const __nv_bfloat16*>(window), accepted, acc_stride, T, S, C,
                                     (long long)(win_stride > 0 ? win_stride : (long long)(3 + T) * C));
  if (e != cudaSuccess) {
    set_error("dfl_gdn_rollback: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_gated_rmsnorm(const void* o, int64_t ldo, const void* z, int64_t ldz, const void* w, void* out,
                                 int64_t ldout, int M, int H, int D, float eps, void* stream) {
  if (M == 0) return DFL_OK;
  if (!o || !z || !w || !out || M < 0 || H <= 0 || D <= 0) {
    set_error("dfl_gated_rmsnorm: bad arguments");
    return DFL_ERR_INVALID;
  }
  const long long items = (long long)M * H;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3((unsigned)((items + 7) / 8)), dim3(256), 0, as_stream(stream), attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gated_rmsnorm_kernel, static_cast<const __nv_bfloat16*>(o), (long long)ldo,
                                     static_cast<const __nv_bfloat16*>(z), (long long)ldz,
                                     static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(out),
                                     (long long)ldout, M, H, D, eps);
  if (e != cudaSuccess) {
    set_error("dfl_gated_rmsnorm: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}
