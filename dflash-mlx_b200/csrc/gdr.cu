// Gated-delta-rule recurrence (Qwen3.5 / Qwen3-Next linear-attention layers).
//
// Per token t, per value head h (key head h / (Hv/Hk)), per value row i:
//   S      <- g_t * S                       (g_t is the decay multiplier, not its log)
//   kv_i    = sum_j S[i,j] k_t[j]
//   delta_i = beta_t * (v_t[i] - kv_i)
//   S[i,:] <- S[i,:] + delta_i * k_t
//   o_t[i]  = sum_j S[i,j] q_t[j]
// State layout [B][Hv][Dv][Dk] fp32 (dflash_mlx/adapters.py:188, the row index is
// the value dimension). This is the recurrence of mlx-lm gated_delta_kernel /
// gated_delta_ops called at custom_qwen35_model.py:452-476, and with o and the
// snapshots switched off it is the state replay of the reference's Metal kernel
// gated_delta_state_update (adapters.py:30-87, 93-135).
//
// B200 design: four lanes per value row, each holding Dk/4 fp32 state elements
// in registers as float4 chunks interleaved across the four lanes (lane c owns
// chunks c, c + 4, ...), so a warp advances 8 value rows per token and each dot
// product is four independent FMA chains plus two shuffles inside the lane group.
// Key, query, value, decay and beta of a 16-token tile are staged in shared
// memory (keys and queries converted to fp32 once). Optional per-token snapshots
// (the state after each token) are written with 16-byte stores so that cache
// rollback to "after a tokens" is a pointer choice instead of a replay. Each
// token's arithmetic is the same whatever T is, so a row advanced inside a
// 16-token verify block and one advanced alone agree bit for bit.
#include "common.cuh"

#include <cstdlib>

namespace dfl {

constexpr int GDR_TT = 16;                    // tokens per staged tile
constexpr int GDR_ROWS = 16;                  // value rows per CTA (every lane layout below)
constexpr int GDR_DEFAULT_LPR = 4;

struct GdrArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* g;
  const float* beta;
  const float* state_in;
  long long state_in_bstride;  // elements between batch entries of state_in
  const int* state_slot;       // nullable: state_in + slot[b] * Hv*Dv*Dk selects a snapshot
  const int* tokens;           // nullable: sequence b advances over min(T, tokens[b * tokens_stride]) tokens
  int tokens_stride;
  float* state_out;
  float* snap;
  __nv_bfloat16* o;
  int B, T, Hk, Hv, Dk, Dv;
};

__device__ __forceinline__ float4 bf16x4_to_float4(uint2 r) {
  return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u), __uint_as_float(r.y << 16),
                     __uint_as_float(r.y & 0xffff0000u));
}

// GDR_LPR lanes per value row; a CTA holds GDR_ROWS rows, so GDR_ROWS * GDR_LPR / 32 warps
template <int DK, int GDR_LPR>
__global__ void __launch_bounds__(GDR_ROWS * GDR_LPR) gdr_kernel(GdrArgs a) {
  constexpr int GDR_WARPS = GDR_ROWS * GDR_LPR / 32;
  (void)GDR_WARPS;
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  constexpr int NCH = DK / (4 * GDR_LPR);  // float4 chunks per lane
  // double-buffered raw tiles: tile i + 1 streams in (cp.async) while tile i is consumed
  __shared__ __align__(16) __nv_bfloat16 sk[2][GDR_TT][DK];
  __shared__ __align__(16) __nv_bfloat16 sq[2][GDR_TT][DK];
  __shared__ __align__(16) __nv_bfloat16 sv[2][GDR_TT][GDR_ROWS];
  __shared__ __align__(16) float sg[2][GDR_TT], sb[2][GDR_TT];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane & (GDR_LPR - 1);
  const int rloc = warp * (32 / GDR_LPR) + (lane / GDR_LPR);  // row inside the CTA
  const int b = blockIdx.z, h = blockIdx.y;
  const int row0 = blockIdx.x * GDR_ROWS;
  const int row = row0 + rloc;
  const int hk = h / (a.Hv / a.Hk);
  const long long hstate = (long long)a.Dv * DK;
  const long long slot_elems = (long long)a.Hv * hstate;
  const bool want_o = a.o != nullptr;

  auto stage = [&](int buf, int t0) {
    const int nt = min(GDR_TT, a.T - t0);
    for (int idx = threadIdx.x; idx < nt * (DK / 8); idx += blockDim.x) {
      const int tt = idx / (DK / 8), cc = idx % (DK / 8);
      const long long off = (((long long)b * a.T + t0 + tt) * a.Hk + hk) * DK + cc * 8;
      cp_async16(smem_u32(&sk[buf][tt][cc * 8]), a.k + off, 16);
      if (want_o) cp_async16(smem_u32(&sq[buf][tt][cc * 8]), a.q + off, 16);
    }
    for (int idx = threadIdx.x; idx < nt * (GDR_ROWS / 8); idx += blockDim.x) {
      const int tt = idx / (GDR_ROWS / 8), cc = idx % (GDR_ROWS / 8);
      cp_async16(smem_u32(&sv[buf][tt][cc * 8]), a.v + (((long long)b * a.T + t0 + tt) * a.Hv + h) * a.Dv + row0 + cc * 8,
                 16);
    }
    for (int tt = threadIdx.x; tt < nt; tt += blockDim.x) {
      const long long gi = ((long long)b * a.T + t0 + tt) * a.Hv + h;
      cp_async4(smem_u32(&sg[buf][tt]), a.g + gi);
      cp_async4(smem_u32(&sb[buf][tt]), a.beta + gi);
    }
  };

  stage(0, 0);
  cp_async_commit();

  const float* sin = a.state_in + b * a.state_in_bstride + (a.state_slot ? (long long)a.state_slot[b] * slot_elems : 0) +
                     h * hstate + (long long)row * DK;
  float4 s[NCH];
#pragma unroll
  for (int j = 0; j < NCH; ++j) s[j] = reinterpret_cast<const float4*>(sin)[j * GDR_LPR + c];

  int buf = 0;
  const int Tb = a.tokens ? max(0, min(a.T, a.tokens[(long long)b * a.tokens_stride])) : a.T;
  for (int t0 = 0; t0 < Tb; t0 += GDR_TT, buf ^= 1) {
    const int nt = min(GDR_TT, Tb - t0);
    if (t0 + GDR_TT < Tb) stage(buf ^ 1, t0 + GDR_TT);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt) {
      const float gt = sg[buf][tt];
      const uint2* kp = reinterpret_cast<const uint2*>(sk[buf][tt]);
      float4 kf[NCH];
      float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        kf[j] = bf16x4_to_float4(kp[j * GDR_LPR + c]);
        s[j].x *= gt;
        s[j].y *= gt;
        s[j].z *= gt;
        s[j].w *= gt;
        p0 += s[j].x * kf[j].x;
        p1 += s[j].y * kf[j].y;
        p2 += s[j].z * kf[j].z;
        p3 += s[j].w * kf[j].w;
      }
      float kv = (p0 + p1) + (p2 + p3);
#pragma unroll
      for (int o = 1; o < GDR_LPR; o <<= 1) kv += __shfl_xor_sync(0xffffffffu, kv, o);
      const float delta = (bf2f(sv[buf][tt][rloc]) - kv) * sb[buf][tt];
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        s[j].x += kf[j].x * delta;
        s[j].y += kf[j].y * delta;
        s[j].z += kf[j].z * delta;
        s[j].w += kf[j].w * delta;
      }
      const int t = t0 + tt;
      if (want_o) {
        const uint2* qp = reinterpret_cast<const uint2*>(sq[buf][tt]);
        float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          const float4 qf = bf16x4_to_float4(qp[j * GDR_LPR + c]);
          y0 += s[j].x * qf.x;
          y1 += s[j].y * qf.y;
          y2 += s[j].z * qf.z;
          y3 += s[j].w * qf.w;
        }
        float y = (y0 + y1) + (y2 + y3);
#pragma unroll
        for (int o = 1; o < GDR_LPR; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (c == 0) a.o[(((long long)b * a.T + t) * a.Hv + h) * a.Dv + row] = f2bf(y);
      }
      if (a.snap) {
        float4* dst = reinterpret_cast<float4*>(a.snap + (((long long)b * a.T + t) * a.Hv + h) * hstate +
                                                (long long)row * DK);
#pragma unroll
        for (int j = 0; j < NCH; ++j) dst[j * GDR_LPR + c] = s[j];
      }
    }
    __syncthreads();  // the buffer just read is refilled two tiles later
  }
  cp_async_wait<0>();
  if (a.state_out) {
    float4* dst = reinterpret_cast<float4*>(a.state_out + ((long long)b * a.Hv + h) * hstate + (long long)row * DK);
#pragma unroll
    for (int j = 0; j < NCH; ++j) dst[j * GDR_LPR + c] = s[j];
  }
}

}  // namespace dfl

using namespace dfl;

// Lanes per value row (4, 8 or 16): more lanes put more warps in flight on the short
// dependent chain of a verify block. A process-wide constant (DFLASH_B200_GDR_LPR sets it
// for tuning), so every call of a session uses the same per-token arithmetic.
static int gdr_lanes_per_row() {
  static int lpr = [] {
    const char* e = getenv("DFLASH_B200_GDR_LPR");
    const int v = e ? atoi(e) : GDR_DEFAULT_LPR;
    return (v == 4 || v == 8 || v == 16) ? v : GDR_DEFAULT_LPR;
  }();
  return lpr;
}

extern "C" int dfl_gdr_recurrence(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                  const float* state_in, int64_t state_in_bstride, const int32_t* state_slot,
                                  float* state_out, float* snapshots, void* o, int B, int T, int Hk, int Hv, int Dk,
                                  int Dv, const int32_t* tokens, int tokens_stride, void* stream) {
  if (B == 0 || T == 0) return DFL_OK;
  if (!k || !v || !g || !beta || !state_in || (o && !q) || B < 0 || T < 0 || Hk <= 0 || Hv <= 0 || Hv % Hk) {
    set_error("dfl_gdr_recurrence: bad arguments");
    return DFL_ERR_INVALID;
  }
  if (Dk != 128 && Dk != 64) {
    set_error("dfl_gdr_recurrence: key head dim %d not supported (64, 128)", Dk);
    return DFL_ERR_UNSUPPORTED;
  }
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(q)) & 15) {
    set_error("dfl_gdr_recurrence: q, k and v must be 16-byte aligned");
    return DFL_ERR_UNSUPPORTED;
  }
  if (Dv % GDR_ROWS) {
    set_error("dfl_gdr_recurrence: value head dim must be a multiple of %d", GDR_ROWS);
    return DFL_ERR_UNSUPPORTED;
  }
  GdrArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.g = g;
  a.beta = beta;
  a.state_in = state_in;
  a.state_in_bstride = state_in_bstride;
  a.state_slot = state_slot;
  a.tokens = tokens;
  a.tokens_stride = tokens_stride;
  a.state_out = state_out;
  a.snap = snapshots;
  a.o = static_cast<__nv_bfloat16*>(o);
  a.B = B;
  a.T = T;
  a.Hk = Hk;
  a.Hv = Hv;
  a.Dk = Dk;
  a.Dv = Dv;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  const int lpr = gdr_lanes_per_row();
  cfg.gridDim = dim3(Dv / GDR_ROWS, Hv, B);
  cfg.blockDim = dim3(GDR_ROWS * lpr);
  cfg.stream = as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (Dk == 128)
    e = lpr == 16 ? cudaLaunchKernelEx(&cfg, gdr_kernel<128, 16>, a)
        : lpr == 8 ? cudaLaunchKernelEx(&cfg, gdr_kernel<128, 8>, a)
                   : cudaLaunchKernelEx(&cfg, gdr_kernel<128, 4>, a);
  else
    e = lpr == 16 ? cudaLaunchKernelEx(&cfg, gdr_kernel<64, 16>, a)
        : lpr == 8 ? cudaLaunchKernelEx(&cfg, gdr_kernel<64, 8>, a)
                   : cudaLaunchKernelEx(&cfg, gdr_kernel<64, 4>, a);
  if (e != cudaSuccess) {
    set_error("dfl_gdr_recurrence: launch failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}
