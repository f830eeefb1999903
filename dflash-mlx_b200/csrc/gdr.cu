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
// B200 design: one warp per value row, each lane holding Dk/32 fp32 state
// elements in registers; the two dot products are warp-shuffle reductions. Key,
// query, value, decay and beta of a 32-token tile are staged in shared memory
// by the whole CTA. Optional per-token snapshots (the state after each token)
// are written with 16-byte stores so that cache rollback to "after a tokens" is
// a pointer choice instead of a replay.
#include "common.cuh"

namespace dfl {

constexpr int GDR_ROWS = 4;  // value rows (warps) per CTA
constexpr int GDR_TT = 32;   // tokens per staged tile

struct GdrArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* g;
  const float* beta;
  const float* state_in;
  long long state_in_bstride;  // elements between batch entries of state_in
  const int* state_slot;       // nullable: state_in + slot[b] * Hv*Dv*Dk selects a snapshot
  float* state_out;
  float* snap;
  __nv_bfloat16* o;
  int B, T, Hk, Hv, Dk, Dv;
};

// a lane's PER contiguous fp32 state values: float4 moves for PER % 4 == 0 (Dk 128),
// float2 for PER == 2 (Dk 64)
template <int PER>
__device__ __forceinline__ void load_state(float (&s)[PER], const float* p) {
  if constexpr (PER % 4 == 0) {
#pragma unroll
    for (int i = 0; i < PER / 4; ++i) {
      const float4 f = reinterpret_cast<const float4*>(p)[i];
      s[4 * i] = f.x;
      s[4 * i + 1] = f.y;
      s[4 * i + 2] = f.z;
      s[4 * i + 3] = f.w;
    }
  } else {
    static_assert(PER % 2 == 0, "state slice must be float2-aligned");
#pragma unroll
    for (int i = 0; i < PER / 2; ++i) {
      const float2 f = reinterpret_cast<const float2*>(p)[i];
      s[2 * i] = f.x;
      s[2 * i + 1] = f.y;
    }
  }
}

template <int PER>
__device__ __forceinline__ void store_state(float* p, const float (&s)[PER]) {
  if constexpr (PER % 4 == 0) {
#pragma unroll
    for (int i = 0; i < PER / 4; ++i)
      reinterpret_cast<float4*>(p)[i] = make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < PER / 2; ++i) reinterpret_cast<float2*>(p)[i] = make_float2(s[2 * i], s[2 * i + 1]);
  }
}

template <int DK>
__global__ void __launch_bounds__(32 * GDR_ROWS) gdr_kernel(GdrArgs a) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  constexpr int PER = DK / 32;
  __shared__ __align__(16) __nv_bfloat16 sk[GDR_TT][DK];
  __shared__ __align__(16) __nv_bfloat16 sq[GDR_TT][DK];
  __shared__ float sv[GDR_TT][GDR_ROWS];
  __shared__ float sg[GDR_TT], sb[GDR_TT];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y;
  const int row0 = blockIdx.x * GDR_ROWS;
  const int row = row0 + warp;
  const int hk = h / (a.Hv / a.Hk);
  const long long hstate = (long long)a.Dv * DK;
  const long long slot_elems = (long long)a.Hv * hstate;

  const float* sin = a.state_in + b * a.state_in_bstride + (a.state_slot ? (long long)a.state_slot[b] * slot_elems : 0) +
                     h * hstate + (long long)row * DK;
  float s[PER];
  load_state<PER>(s, sin + lane * PER);

  for (int t0 = 0; t0 < a.T; t0 += GDR_TT) {
    const int nt = min(GDR_TT, a.T - t0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < nt * (DK / 8); idx += blockDim.x) {
      const int tt = idx / (DK / 8), c = idx % (DK / 8);
      const long long off = (((long long)b * a.T + t0 + tt) * a.Hk + hk) * DK + c * 8;
      *reinterpret_cast<uint4*>(&sk[tt][c * 8]) = *reinterpret_cast<const uint4*>(a.k + off);
      if (a.o) *reinterpret_cast<uint4*>(&sq[tt][c * 8]) = *reinterpret_cast<const uint4*>(a.q + off);
    }
    for (int idx = threadIdx.x; idx < nt * GDR_ROWS; idx += blockDim.x) {
      const int tt = idx / GDR_ROWS, r = idx % GDR_ROWS;
      sv[tt][r] = bf2f(a.v[(((long long)b * a.T + t0 + tt) * a.Hv + h) * a.Dv + row0 + r]);
    }
    for (int tt = threadIdx.x; tt < nt; tt += blockDim.x) {
      const long long gi = ((long long)b * a.T + t0 + tt) * a.Hv + h;
      sg[tt] = a.g[gi];
      sb[tt] = a.beta[gi];
    }
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt) {
      float kf[PER];
      {
        const __nv_bfloat16* kp = &sk[tt][lane * PER];
#pragma unroll
        for (int i = 0; i < PER; ++i) kf[i] = bf2f(kp[i]);
      }
      const float gt = sg[tt];
      float kv = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        s[i] *= gt;
        kv += s[i] * kf[i];
      }
      kv = warp_sum(kv);
      const float delta = (sv[tt][warp] - kv) * sb[tt];
#pragma unroll
      for (int i = 0; i < PER; ++i) s[i] += kf[i] * delta;
      const int t = t0 + tt;
      if (a.o) {
        const __nv_bfloat16* qp = &sq[tt][lane * PER];
        float y = 0.f;
#pragma unroll
        for (int i = 0; i < PER; ++i) y += s[i] * bf2f(qp[i]);
        y = warp_sum(y);
        if (lane == 0) a.o[(((long long)b * a.T + t) * a.Hv + h) * a.Dv + row] = f2bf(y);
      }
      if (a.snap) {
        store_state<PER>(a.snap + (((long long)b * a.T + t) * a.Hv + h) * hstate + (long long)row * DK + lane * PER,
                         s);
      }
    }
  }
  if (a.state_out) {
    store_state<PER>(a.state_out + ((long long)b * a.Hv + h) * hstate + (long long)row * DK + lane * PER, s);
  }
}

}  // namespace dfl

using namespace dfl;

extern "C" int dfl_gdr_recurrence(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                  const float* state_in, int64_t state_in_bstride, const int32_t* state_slot,
                                  float* state_out, float* snapshots, void* o, int B, int T, int Hk, int Hv, int Dk,
                                  int Dv, void* stream) {
  if (B == 0 || T == 0) return DFL_OK;
  if (!k || !v || !g || !beta || !state_in || (o && !q) || B < 0 || T < 0 || Hk <= 0 || Hv <= 0 || Hv % Hk) {
    set_error("dfl_gdr_recurrence: bad arguments");
    return DFL_ERR_INVALID;
  }
  if (Dk != 128 && Dk != 64) {
    set_error("dfl_gdr_recurrence: key head dim %d not supported (64, 128)", Dk);
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
  cfg.gridDim = dim3(Dv / GDR_ROWS, Hv, B);
  cfg.blockDim = dim3(32 * GDR_ROWS);
  cfg.stream = as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = Dk == 128 ? cudaLaunchKernelEx(&cfg, gdr_kernel<128>, a) : cudaLaunchKernelEx(&cfg, gdr_kernel<64>, a);
  if (e != cudaSuccess) {
    set_error("dfl_gdr_recurrence: launch failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}
