// Weight-streaming bf16 GEMM for the 16-token verify/draft blocks.
//
//   Y[M, N] = X[M, K] . W[N, K]^T   (fp32 accumulate) + fused epilogue
//
// Replaces the mlx-lm nn.Linear calls inside the Qwen3 / DFlash layers
// (reference: dflash_mlx/draft.py:75-98 q/k/v/o projections, mlx-lm qwen3 MLP
// used at draft.py:13, adapters.py:264-271 lm_head) for the decode-shaped
// case where M is a multiple of 16 rows and the cost is streaming W from HBM.
//
// Design (B200): each CTA owns a 16-row x 64-column output tile and a contiguous
// range of K blocks (split-K chosen from N and K only, never from M, so every
// output row is computed with the same reduction order whatever the batch is:
// the lossless spec-decode == plain-greedy property relies on this). W tiles
// are streamed with 16-byte cp.async into a 6-stage XOR-swizzled ring, the four
// warps each take one 16-wide k slice of every stage (mma.sync m16n8k16), the
// warp partials are reduced in shared memory in a fixed order, and split-K
// partials are reduced by the last-arriving CTA of a tile, again in split order.
#include "common.cuh"

namespace dfl {

constexpr int GS_BM = 16;
constexpr int GS_BN = 64;
constexpr int GS_BK = 64;
constexpr int GS_STAGES = 6;
constexpr int GS_THREADS = 128;
constexpr int GS_W_STAGE = GS_BN * GS_BK;  // bf16 elements
constexpr int GS_X_STAGE = GS_BM * GS_BK;
constexpr int GS_SMEM = GS_STAGES * (GS_W_STAGE + GS_X_STAGE) * 2;
// Split-K arrival counters live in a fixed region at the start of the workspace so
// that the partials of one call can never land on another call's counters.
constexpr int GS_MAX_COUNTERS = 1 << 17;
constexpr size_t GS_COUNTER_BYTES = (size_t)GS_MAX_COUNTERS * sizeof(int);

struct GemmStreamArgs {
  const __nv_bfloat16* x;
  long long ldx;
  const __nv_bfloat16* w;
  const __nv_bfloat16* res;
  long long ldr;
  __nv_bfloat16* y;
  long long ldy;
  __nv_bfloat16* y2;  // optional second destination (hidden-state tap)
  long long ldy2;
  float2* argmax;  // [M][n_tiles] (value, index-as-float-bits)
  float* partial;  // [m_tiles][n_tiles][splits][16*64]
  int* counters;   // [m_tiles][n_tiles]
  int M, N, K;
  int n_tiles, splits, kblocks;
};

// swizzled element offset of (row, 16B chunk c) in a 64-wide bf16 tile
__device__ __forceinline__ int swz(int row, int c) { return row * 64 + ((c ^ (row & 7)) << 3); }

template <int EPI>
__global__ void __launch_bounds__(GS_THREADS) gemm_stream_kernel(GemmStreamArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __nv_bfloat16* sW = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sX = sW + GS_STAGES * GS_W_STAGE;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int ntile = blockIdx.x;
  const int split = blockIdx.y;
  const int mtile = blockIdx.z;
  const int n0 = ntile * GS_BN;
  const int m0 = mtile * GS_BM;

  // contiguous k-block range of this split
  const int kb_begin = (int)(((long long)split * a.kblocks) / a.splits);
  const int kb_end = (int)(((long long)(split + 1) * a.kblocks) / a.splits);
  const int nkb = kb_end - kb_begin;
  grid_dependency_launch_dependents();

  // Weights do not depend on the upstream kernel: start streaming them before
  // waiting on the grid dependency (programmatic dependent launch).
  auto load_w = [&](int slot, int kb) {
    const int k0 = kb * GS_BK;
    __nv_bfloat16* dst = sW + slot * GS_W_STAGE;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + i * GS_THREADS;
      const int row = q >> 3, c = q & 7;
      const int n = n0 + row;
      const __nv_bfloat16* src = a.w + (long long)(n < a.N ? n : 0) * a.K + k0 + c * 8;
      cp_async16(smem_u32(dst + swz(row, c)), src, n < a.N ? 16 : 0);
    }
  };
  auto load_x = [&](int slot, int kb) {
    const int k0 = kb * GS_BK;
    __nv_bfloat16* dst = sX + slot * GS_X_STAGE;
    const int row = tid >> 3, c = tid & 7;
    const int m = m0 + row;
    const __nv_bfloat16* src = a.x + (long long)(m < a.M ? m : 0) * a.ldx + k0 + c * 8;
    cp_async16(smem_u32(dst + swz(row, c)), src, m < a.M ? 16 : 0);
  };

  // Prologue: weights for the first stages go out before the dependency wait.
#pragma unroll
  for (int s = 0; s < GS_STAGES - 1; ++s)
    if (s < nkb) load_w(s, kb_begin + s);
  grid_dependency_wait();
#pragma unroll
  for (int s = 0; s < GS_STAGES - 1; ++s) {
    if (s < nkb) load_x(s, kb_begin + s);
    cp_async_commit();
  }

  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;

  for (int it = 0; it < nkb; ++it) {
    cp_async_wait<GS_STAGES - 2>();
    __syncthreads();
    {
      const int nxt = it + GS_STAGES - 1;
      if (nxt < nkb) {
        load_w(nxt % GS_STAGES, kb_begin + nxt);
        load_x(nxt % GS_STAGES, kb_begin + nxt);
      }
      cp_async_commit();
    }
    const int slot = it % GS_STAGES;
    const __nv_bfloat16* tW = sW + slot * GS_W_STAGE;
    const __nv_bfloat16* tX = sX + slot * GS_X_STAGE;
    // this warp's 16-wide k slice: 16B chunks 2*warp and 2*warp+1
    uint32_t af[4];
    {
      const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = 2 * warp + (lane >> 4);
      ldmatrix_x4(smem_u32(tX + swz(row, c)), af[0], af[1], af[2], af[3]);
    }
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      const int row = nb * 16 + (lane & 7) + (lane >> 4) * 8;
      const int c = 2 * warp + ((lane >> 3) & 1);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(smem_u32(tW + swz(row, c)), b0, b1, b2, b3);
      mma_bf16_16816(acc[2 * nb], af, b0, b1);
      mma_bf16_16816(acc[2 * nb + 1], af, b2, b3);
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // Reduce the four warp partials in a fixed order into red[16][64].
  float* wpart = reinterpret_cast<float*>(smem_raw);  // [4][16][64] = 16 KB (ring is idle now)
  {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = j * 8 + 2 * t;
      float* p = wpart + warp * 1024;
      p[g * 64 + col] = acc[j][0];
      p[g * 64 + col + 1] = acc[j][1];
      p[(g + 8) * 64 + col] = acc[j][2];
      p[(g + 8) * 64 + col + 1] = acc[j][3];
    }
  }
  __syncthreads();
  float* red = wpart + 4 * 1024;  // [16][64]
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = tid + i * GS_THREADS;
    red[e] = ((wpart[e] + wpart[1024 + e]) + wpart[2048 + e]) + wpart[3072 + e];
  }
  __syncthreads();

  if (a.splits > 1) {
    __shared__ int is_last;
    const int tile_id = mtile * a.n_tiles + ntile;
    float* mine = a.partial + ((long long)tile_id * a.splits + split) * 1024;
#pragma unroll
    for (int i = 0; i < 8; ++i) mine[tid + i * GS_THREADS] = red[tid + i * GS_THREADS];
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(a.counters + tile_id, 1);
      is_last = (prev == a.splits - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* base = a.partial + (long long)tile_id * a.splits * 1024;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + i * GS_THREADS;
      float s = 0.f;
      for (int sp = 0; sp < a.splits; ++sp) s += __ldcg(base + (long long)sp * 1024 + e);
      red[e] = s;
    }
    if (tid == 0) a.counters[tile_id] = 0;  // ready for the next launch / graph replay
    __syncthreads();
  }

  // Epilogues
  if constexpr (EPI == DFL_EPI_STORE || EPI == DFL_EPI_RESIDUAL) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + i * GS_THREADS;
      const int r = e >> 6, c = e & 63;
      const int m = m0 + r, n = n0 + c;
      if (m < a.M && n < a.N) {
        float v = red[e];
        if constexpr (EPI == DFL_EPI_RESIDUAL) v = bf2f(a.res[(long long)m * a.ldr + n]) + round_bf16(v);
        const __nv_bfloat16 o = f2bf(v);
        a.y[(long long)m * a.ldy + n] = o;
        if (a.y2) a.y2[(long long)m * a.ldy2 + n] = o;
      }
    }
  } else if constexpr (EPI == DFL_EPI_SILU_MUL) {
    // tile columns [0,32) are gate rows, [32,64) the matching up rows
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * GS_THREADS;
      const int r = e >> 5, j = e & 31;
      const int m = m0 + r, n = ntile * 32 + j;
      if (m < a.M && n0 + j < a.N) {
        const float gt = round_bf16(red[r * 64 + j]);
        const float up = round_bf16(red[r * 64 + 32 + j]);
        const float act = round_bf16(gt / (1.f + __expf(-gt)));
        a.y[(long long)m * a.ldy + n] = f2bf(act * up);
      }
    }
  } else if constexpr (EPI == DFL_EPI_ARGMAX) {
    // per row: max of bf16-rounded logits over the tile, lowest index on ties
    const int r = tid >> 3, sub = tid & 7;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      const int c = sub * 8 + c8;
      const int n = n0 + c;
      if (n < a.N) {
        const float v = round_bf16(red[r * 64 + c]);
        if (v > best) { best = v; bidx = n; }
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
      if (ob > best || (ob == best && oi < bidx)) { best = ob; bidx = oi; }
    }
    const int m = m0 + r;
    if (sub == 0 && m < a.M) a.argmax[(long long)m * a.n_tiles + ntile] = make_float2(best, __int_as_float(bidx));
  }
}

struct StreamPlan {
  int n_tiles, m_tiles, splits, kblocks;
};

static StreamPlan plan_stream(int M, int N, int K) {
  StreamPlan p;
  p.n_tiles = (N + GS_BN - 1) / GS_BN;
  p.m_tiles = (M + GS_BM - 1) / GS_BM;
  p.kblocks = K / GS_BK;
  // Split K so that about three CTAs per SM (148 SMs) stream weights at once.
  // Depends on N and K only (row-invariance of the reduction order).
  const int target = 148 * 3;
  int s = (target + p.n_tiles - 1) / p.n_tiles;
  const int max_s = p.kblocks / 4 > 0 ? p.kblocks / 4 : 1;  // >= 4 k-blocks per split
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  p.splits = s;
  return p;
}

}  // namespace dfl

using namespace dfl;

extern "C" size_t dfl_gemm_workspace_bytes(int M, int N, int K, int epilogue) {
  (void)epilogue;
  if (M <= 0 || N <= 0 || K <= 0 || K % GS_BK) return 0;
  StreamPlan p = plan_stream(M, N, K);
  if (p.splits == 1) return 0;
  const size_t tiles = (size_t)p.m_tiles * p.n_tiles;
  return GS_COUNTER_BYTES + tiles * p.splits * 1024 * sizeof(float);
}

extern "C" int dfl_gemm_argmax_tiles(int N) { return (N + GS_BN - 1) / GS_BN; }

extern "C" int dfl_gemm_bf16(const void* x, int64_t ldx, const void* w, int M, int N, int K, int epilogue,
                             const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                             void* argmax_partials, void* workspace, size_t workspace_bytes, void* stream) {
  if (M == 0) return DFL_OK;
  if (!x || !w || M < 0 || N <= 0 || K <= 0) {
    set_error("dfl_gemm_bf16: null pointer or bad shape M=%d N=%d K=%d", M, N, K);
    return DFL_ERR_INVALID;
  }
  if (K % GS_BK || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) {
    set_error("dfl_gemm_bf16: K must be a multiple of 64 and x/w 16-byte aligned with ldx %% 8 == 0 (K=%d ldx=%lld)",
              K, (long long)ldx);
    return DFL_ERR_UNSUPPORTED;
  }
  if (epilogue == DFL_EPI_ARGMAX) {
    if (!argmax_partials) { set_error("dfl_gemm_bf16: argmax epilogue needs argmax_partials"); return DFL_ERR_INVALID; }
  } else if (!y) {
    set_error("dfl_gemm_bf16: y is null");
    return DFL_ERR_INVALID;
  }
  if (epilogue == DFL_EPI_RESIDUAL && !residual) {
    set_error("dfl_gemm_bf16: residual epilogue needs a residual pointer");
    return DFL_ERR_INVALID;
  }
  if (epilogue == DFL_EPI_SILU_MUL && N % GS_BN) {
    set_error("dfl_gemm_bf16: silu-mul epilogue needs N %% 64 == 0 (packed gate/up), N=%d", N);
    return DFL_ERR_UNSUPPORTED;
  }
  StreamPlan p = plan_stream(M, N, K);
  GemmStreamArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.y2 = static_cast<__nv_bfloat16*>(y2);
  a.ldy2 = ldy2;
  a.argmax = static_cast<float2*>(argmax_partials);
  a.M = M;
  a.N = N;
  a.K = K;
  a.n_tiles = p.n_tiles;
  a.splits = p.splits;
  a.kblocks = p.kblocks;
  a.counters = nullptr;
  a.partial = nullptr;
  if (p.splits > 1) {
    const size_t need = dfl_gemm_workspace_bytes(M, N, K, epilogue);
    if (!workspace || workspace_bytes < need) {
      set_error("dfl_gemm_bf16: workspace too small (%zu < %zu bytes)", workspace_bytes, need);
      return DFL_ERR_WORKSPACE;
    }
    const size_t tiles = (size_t)p.m_tiles * p.n_tiles;
    if (tiles > (size_t)GS_MAX_COUNTERS) {
      set_error("dfl_gemm_bf16: %zu output tiles exceed the split-K counter region (%d)", tiles, GS_MAX_COUNTERS);
      return DFL_ERR_UNSUPPORTED;
    }
    a.counters = static_cast<int*>(workspace);
    a.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + GS_COUNTER_BYTES);
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_tiles, p.splits, p.m_tiles);
  cfg.blockDim = dim3(GS_THREADS);
  cfg.dynamicSmemBytes = GS_SMEM;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;

  cudaError_t err;
  switch (epilogue) {
#define DFL_LAUNCH(E)                                                                          \
  case E: {                                                                                    \
    static bool init = false;                                                                  \
    if (!init) {                                                                               \
      cudaFuncSetAttribute(gemm_stream_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           GS_SMEM);                                                           \
      init = true;                                                                             \
    }                                                                                          \
    err = cudaLaunchKernelEx(&cfg, gemm_stream_kernel<E>, a);                                  \
    break;                                                                                     \
  }
    DFL_LAUNCH(DFL_EPI_STORE)
    DFL_LAUNCH(DFL_EPI_RESIDUAL)
    DFL_LAUNCH(DFL_EPI_SILU_MUL)
    DFL_LAUNCH(DFL_EPI_ARGMAX)
#undef DFL_LAUNCH
    default:
      set_error("dfl_gemm_bf16: unknown epilogue %d", epilogue);
      return DFL_ERR_INVALID;
  }
  if (err != cudaSuccess) {
    set_error("dfl_gemm_bf16: launch failed: %s", cudaGetErrorString(err));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}
