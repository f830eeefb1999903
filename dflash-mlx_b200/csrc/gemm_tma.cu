// Persistent TMA-fed weight-streaming GEMM for the 16-token decode blocks.
//
//   Y[M, N] = Xn[M, K] . W[N, K]^T   (fp32 accumulate) + fused epilogue
//   Xn      = X, or RMSNorm(X) with weight norm_w when the prologue is enabled
//
// Replaces the nn.Linear (and the RMSNorm feeding it) of the verify / draft
// forward: mlx-lm qwen3 Attention / MLP projections driven from
// adapters.py:611-631, DFlashAttention q/k/v/o (draft.py:75-98, 118-159), the
// draft fc + hidden_norm (draft.py:196-201, 217) and lm_head_logits /
// lm_head_argmax (adapters.py:264-271, 606-609).
//
// B200 design
//  * One CTA per SM (grid = 148 per 16-row tile of X), persistent over a
//    contiguous range of work units; a unit is one 64-row x 64-k tile of W. The
//    ranges are an even split of the units of one 16-row tile, so every SM streams
//    the same number of weight bytes and there is no tail wave.
//  * A producer warp issues 2-D TMA loads (128-byte swizzle, evict-first L2 hint)
//    into an 8-stage mbarrier ring; the first stages of W are issued BEFORE
//    griddepcontrol.wait, so under programmatic dependent launch a GEMM streams its
//    weights while the previous kernel is still finishing.
//  * Four consumer warps run mma.sync m16n8k16 (one 16-wide k slice each per
//    stage). M = 16 tokens is far below a tcgen05 tile, and the tensor pipe is
//    idle >95% of the time here: the kernel is bound by HBM.
//  * Optional fused RMSNorm prologue: the row sum-of-squares arrives as per-64-
//    column partials written by the epilogue that produced X (or by the embedding
//    gather); consumers reduce them in a fixed order and rescale each X stage in
//    shared memory before the MMAs.
//  * Tiles cut by a range boundary are reduced by the last-arriving CTA in a fixed
//    segment order. Split points depend on N and K only, so a row's result is
//    bit-identical whatever M is (spec-verify rows == plain-decode rows).
#include "tma_util.cuh"

#include <mutex>
#include <unordered_map>

namespace dfl {

static __device__ int g_device_error = 0;

int* device_error_word() {
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

constexpr int TG_NT = 64;
constexpr int TG_BK = 128;  // k per stage: two 64-column TMA boxes (128-byte swizzle rows)
constexpr int TG_BM = 16;
constexpr int TG_STAGES = 4;
constexpr int TG_NORM_MAX_K = 8192;  // fused-RMSNorm weights staged in shared memory
constexpr int TG_GRID = 148;  // work split over the B200's SM count (fixed: part of the reduction order)
constexpr int TG_CONSUMERS = 4;
constexpr int TG_THREADS = 32 * (TG_CONSUMERS + 1);
constexpr int TG_W_HALF = TG_NT * 64 * 2;  // one 64-row x 64-k box: 8 KB
constexpr int TG_X_HALF = TG_BM * 64 * 2;  // one 16-row x 64-k box: 2 KB
constexpr int TG_W_BYTES = 2 * TG_W_HALF;
constexpr int TG_X_BYTES = 2 * TG_X_HALF;
constexpr int TG_OFF_X = TG_STAGES * TG_W_BYTES;
constexpr int TG_OFF_WPART = TG_OFF_X + TG_STAGES * TG_X_BYTES;
constexpr int TG_OFF_RED = TG_OFF_WPART + TG_CONSUMERS * TG_BM * TG_NT * 4;
constexpr int TG_OFF_BAR = TG_OFF_RED + TG_BM * TG_NT * 4;
constexpr int TG_OFF_NORM = TG_OFF_BAR + 2 * TG_STAGES * 8;  // K bf16 norm weights follow when fused
constexpr int TG_SMEM_BASE = TG_OFF_NORM + 1024;                // + alignment slack
constexpr int TG_MAX_COUNTERS = 1 << 17;
constexpr size_t TG_COUNTER_BYTES = (size_t)TG_MAX_COUNTERS * sizeof(int);

struct TgArgs {
  const __nv_bfloat16* res;
  long long ldr;
  __nv_bfloat16* y;
  long long ldy;
  __nv_bfloat16* y2;
  long long ldy2;
  float2* argmax;      // [M][n_tiles]
  float* partial;      // [m_tiles][grid1][2][16*64]
  int* counters;       // [m_tiles * n_tiles]
  const __nv_bfloat16* norm_w;  // fused RMSNorm weight (nullable: no prologue)
  const float* sumsq_in;        // [M][n_parts] row sum-of-squares partials of X
  int n_parts;
  float eps;
  float* sumsq_out;  // [M][n_tiles] partials of the bf16 output (nullable)
  int* err;  // device error word
  int M, N, K, n_tiles, kb;
  long long U1;  // units of one 16-row tile = n_tiles * kb
  int grid1;     // CTAs per 16-row tile
};

__device__ __forceinline__ int tg_swz(int row, int c) { return row * 64 + ((c ^ (row & 7)) << 3); }

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(32 * TG_CONSUMERS)); }

// CTA (within one 16-row tile) that owns unit u: max c with floor(c*U/G) <= u.
__device__ __forceinline__ int unit_owner(long long u, long long U, int G) {
  return (int)(((u + 1) * G + U - 1) / U) - 1;
}

template <int EPI>
__device__ void tg_epilogue(const TgArgs& a, const float* red, int mt, int nt, int ct) {
  const int m0 = mt * TG_BM, n0 = nt * TG_NT;
  if constexpr (EPI == DFL_EPI_STORE || EPI == DFL_EPI_RESIDUAL) {
    const int r = ct >> 3, c8 = (ct & 7) * 8;
    const int m = m0 + r, n = n0 + c8;
    float ss = 0.f;
    if (m < a.M && n < a.N) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = red[r * TG_NT + c8 + e];
      if constexpr (EPI == DFL_EPI_RESIDUAL) {
        const uint4 rv = *reinterpret_cast<const uint4*>(a.res + (long long)m * a.ldr + n);
        const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = bf2f(re[e]) + round_bf16(v[e]);
      }
      uint4 o;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        oe[e] = f2bf(v[e]);
        const float q = bf2f(oe[e]);
        ss += q * q;
      }
      *reinterpret_cast<uint4*>(a.y + (long long)m * a.ldy + n) = o;
      if (a.y2) *reinterpret_cast<uint4*>(a.y2 + (long long)m * a.ldy2 + n) = o;
    }
    if (a.sumsq_out) {
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      ss += __shfl_xor_sync(0xffffffffu, ss, 4);
      if ((ct & 7) == 0 && m < a.M) a.sumsq_out[(long long)m * a.n_tiles + nt] = ss;
    }
  } else if constexpr (EPI == DFL_EPI_SILU_MUL) {
    // tile columns [0,32) gate rows, [32,64) the matching up rows -> 32 outputs per row
    const int r = ct >> 3, j4 = (ct & 7) * 4;
    const int m = m0 + r;
    if (m < a.M && n0 + j4 < a.N) {
      uint2 o;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float gt = round_bf16(red[r * TG_NT + j4 + e]);
        const float up = round_bf16(red[r * TG_NT + 32 + j4 + e]);
        const float act = round_bf16(gt / (1.f + __expf(-gt)));
        oe[e] = f2bf(act * up);
      }
      *reinterpret_cast<uint2*>(a.y + (long long)m * a.ldy + nt * 32 + j4) = o;
    }
  } else if constexpr (EPI == DFL_EPI_ARGMAX) {
    const int r = ct >> 3, sub = ct & 7;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      const int c = sub * 8 + c8;
      const int n = n0 + c;
      if (n < a.N) {
        const float v = round_bf16(red[r * TG_NT + c]);
        if (v > best) { best = v; bidx = n; }
      }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
      if (ob > best || (ob == best && oi < bidx)) { best = ob; bidx = oi; }
    }
    const int m = m0 + r;
    if (sub == 0 && m < a.M) a.argmax[(long long)m * a.n_tiles + nt] = make_float2(best, __int_as_float(bidx));
  }
}

template <int EPI>
__global__ void __launch_bounds__(TG_THREADS, 1)
    gemm_tma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, TgArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __nv_bfloat16* sW = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sX = reinterpret_cast<__nv_bfloat16*>(smem + TG_OFF_X);
  float* wpart = reinterpret_cast<float*>(smem + TG_OFF_WPART);
  float* red = reinterpret_cast<float*>(smem + TG_OFF_RED);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TG_OFF_BAR);
  uint64_t* empty = full + TG_STAGES;
  __shared__ float s_inv[TG_BM];
  __shared__ int s_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x / a.grid1;
  const int c = blockIdx.x % a.grid1;
  const long long u0 = (long long)c * a.U1 / a.grid1;
  const long long u1 = (long long)(c + 1) * a.U1 / a.grid1;
  const int n_units = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < TG_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], TG_CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  grid_dependency_launch_dependents();

  if (warp == TG_CONSUMERS) {
    // ---------------- producer ----------------
    if (lane == 0 && n_units > 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const int pre = n_units < TG_STAGES ? n_units : TG_STAGES;
      auto load_w = [&](int s, int nt, int j) {
        unsigned char* d = smem + s * TG_W_BYTES;
        tma_load_2d(&wmap, &full[s], d, j * TG_BK, nt * TG_NT, pol_w);
        tma_load_2d(&wmap, &full[s], d + TG_W_HALF, j * TG_BK + 64, nt * TG_NT, pol_w);
      };
      auto load_x = [&](int s, int j) {
        unsigned char* d = smem + TG_OFF_X + s * TG_X_BYTES;
        tma_load_2d(&xmap, &full[s], d, j * TG_BK, mt * TG_BM, pol_x);
        tma_load_2d(&xmap, &full[s], d + TG_X_HALF, j * TG_BK + 64, mt * TG_BM, pol_x);
      };
      for (int i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        mbar_expect_tx(&full[i], TG_W_BYTES + TG_X_BYTES);
        load_w(i, (int)(u / a.kb), (int)(u % a.kb));
      }
      grid_dependency_wait();  // X is produced by the previous kernel
      for (int i = 0; i < pre; ++i) load_x(i, (int)((u0 + i) % a.kb));
      for (int i = pre; i < n_units; ++i) {
        const int s = i % TG_STAGES;
        if (!mbar_wait(&empty[s], ((i / TG_STAGES) & 1) ^ 1, 101, a.err)) break;
        const long long u = u0 + i;
        mbar_expect_tx(&full[s], TG_W_BYTES + TG_X_BYTES);
        load_w(s, (int)(u / a.kb), (int)(u % a.kb));
        load_x(s, (int)(u % a.kb));
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int ct = threadIdx.x;  // 0..127
  const bool norm = a.norm_w != nullptr;
  __nv_bfloat16* s_nw = reinterpret_cast<__nv_bfloat16*>(smem + TG_OFF_NORM);
  if (norm)  // norm weights are parameters (not produced upstream): stage them before the wait
    for (int k = ct * 8; k < a.K; k += 128 * 8)
      *reinterpret_cast<uint4*>(s_nw + k) = *reinterpret_cast<const uint4*>(a.norm_w + k);
  grid_dependency_wait();
  if (norm && ct < TG_BM) {
    const int m = mt * TG_BM + ct;
    float ss = 0.f;
    if (m < a.M)
      for (int p = 0; p < a.n_parts; ++p) ss += a.sumsq_in[(long long)m * a.n_parts + p];
    s_inv[ct] = rsqrtf(ss / (float)a.K + a.eps);
  }
  if (norm) consumer_sync();

  float acc[8][4];
  bool ok = true;
  for (int i = 0; i < n_units && ok; ++i) {
    const long long u = u0 + i;
    const int nt = (int)(u / a.kb), j = (int)(u % a.kb);
    const int s = i % TG_STAGES;
    if (i == 0 || j == 0) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[q][e] = 0.f;
    }
    if (!mbar_wait(&full[s], (i / TG_STAGES) & 1, 102, a.err)) {
      ok = false;
      break;
    }
    __nv_bfloat16* tX = sX + s * (TG_X_BYTES / 2);
    const __nv_bfloat16* tW = sW + s * (TG_W_BYTES / 2);
    if (norm) {
      // rescale this thread's two 16-byte chunks of the X stage: xn = bf16(w * x * inv_rms)
      const int row = ct >> 3, cc = ct & 7;
      const float inv = s_inv[row];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        __nv_bfloat16* p = tX + hf * (TG_X_HALF / 2) + tg_swz(row, cc);
        uint4 xv = *reinterpret_cast<uint4*>(p);
        const uint4 wv = *reinterpret_cast<const uint4*>(s_nw + j * TG_BK + hf * 64 + cc * 8);
        __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) xe[e] = f2bf(bf2f(we[e]) * (bf2f(xe[e]) * inv));
        *reinterpret_cast<uint4*>(p) = xv;
      }
      consumer_sync();
    }
    // this warp's k16 slices: warp and warp + 4 (one per 64-column half)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const __nv_bfloat16* hX = tX + hf * (TG_X_HALF / 2);
      const __nv_bfloat16* hW = tW + hf * (TG_W_HALF / 2);
      uint32_t af[4];
      {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int cc = 2 * warp + (lane >> 4);
        ldmatrix_x4(smem_u32(hX + tg_swz(row, cc)), af[0], af[1], af[2], af[3]);
      }
#pragma unroll
      for (int nb = 0; nb < 4; ++nb) {
        const int row = nb * 16 + (lane & 7) + (lane >> 4) * 8;
        const int cc = 2 * warp + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_u32(hW + tg_swz(row, cc)), b0, b1, b2, b3);
        mma_bf16_16816(acc[2 * nb], af, b0, b1);
        mma_bf16_16816(acc[2 * nb + 1], af, b2, b3);
      }
    }
    // release the stage (generic-proxy writes of the norm prologue must be ordered
    // before the next TMA write into it)
    if (norm) fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool seg_end = (j == a.kb - 1) || (i == n_units - 1);
    if (!seg_end) continue;
    // -------- end of this CTA's segment of tile nt: reduce warps in a fixed order --------
    {
      const int g = lane >> 2, t = lane & 3;
      float* p = wpart + warp * (TG_BM * TG_NT);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int col = q * 8 + 2 * t;
        p[g * TG_NT + col] = acc[q][0];
        p[g * TG_NT + col + 1] = acc[q][1];
        p[(g + 8) * TG_NT + col] = acc[q][2];
        p[(g + 8) * TG_NT + col + 1] = acc[q][3];
      }
    }
    consumer_sync();
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = ct + q * 128;
      red[e] = ((wpart[e] + wpart[1024 + e]) + wpart[2048 + e]) + wpart[3072 + e];
    }
    consumer_sync();
    const long long tu0 = (long long)nt * a.kb, tu1 = tu0 + a.kb - 1;
    const int c_first = unit_owner(tu0, a.U1, a.grid1), c_last = unit_owner(tu1, a.U1, a.grid1);
    bool do_epi = true;
    if (c_first != c_last) {
      const int tile_id = mt * a.n_tiles + nt;
      const int my_first_tile = (int)(u0 / a.kb);
      const int slot = (nt == my_first_tile) ? 0 : 1;
      float* mine = a.partial + (((long long)mt * a.grid1 + c) * 2 + slot) * (TG_BM * TG_NT);
#pragma unroll
      for (int q = 0; q < 8; ++q) mine[ct + q * 128] = red[ct + q * 128];
      __threadfence();
      consumer_sync();
      if (ct == 0) {
        const int prev = atomicAdd(a.counters + tile_id, 1);
        s_flag = (prev == c_last - c_first);
      }
      consumer_sync();
      do_epi = s_flag != 0;
      if (do_epi) {
        __threadfence();
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int e = ct + q * 128;
          float sum = 0.f;
          for (int cs = c_first; cs <= c_last; ++cs) {
            const long long cs_u0 = (long long)cs * a.U1 / a.grid1;
            const int sl = (nt == (int)(cs_u0 / a.kb)) ? 0 : 1;
            sum += __ldcg(a.partial + (((long long)mt * a.grid1 + cs) * 2 + sl) * (TG_BM * TG_NT) + e);
          }
          red[e] = sum;
        }
        if (ct == 0) a.counters[tile_id] = 0;  // ready for the next launch / graph replay
        consumer_sync();
      }
    }
    if (do_epi) tg_epilogue<EPI>(a, red, mt, nt, ct);
    consumer_sync();  // red / wpart are reused by the next segment
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor-map cache and launch
// ---------------------------------------------------------------------------
struct MapKey {
  const void* base;
  uint64_t rows, cols, ld;
  uint32_t box_rows, box_cols;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows &&
           box_cols == o.box_cols;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.base);
    h ^= std::hash<uint64_t>()(k.rows * 1000003ull + k.cols * 31ull + k.ld) + 0x9e3779b97f4a7c15ull + (h << 6);
    h ^= std::hash<uint64_t>()(((uint64_t)k.box_rows << 32) | k.box_cols) + (h << 6) + (h >> 2);
    return h;
  }
};

static std::mutex g_map_mu;
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash>* g_maps = nullptr;
static PFN_cuTensorMapEncodeTiled g_encode = nullptr;

const CUtensorMap* tensor_map_2d_bf16(const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                                      uint32_t box_rows, uint32_t box_cols) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  if (!g_maps) g_maps = new std::unordered_map<MapKey, CUtensorMap, MapKeyHash>();
  MapKey key{base, rows, cols, ld, box_rows, box_cols};
  auto it = g_maps->find(key);
  if (it != g_maps->end()) return &it->second;
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      set_error("cuTensorMapEncodeTiled is not available from the driver");
      return nullptr;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for rows=%llu cols=%llu ld=%llu", (int)r,
              (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)ld);
    return nullptr;
  }
  if (g_maps->size() > 4096) g_maps->clear();
  auto res = g_maps->emplace(key, map);
  return &res.first->second;
}

struct TgPlan {
  int n_tiles, m_tiles, kb, grid1;
  long long U1;
};

static TgPlan tg_plan(int M, int N, int K) {
  TgPlan p;
  p.n_tiles = (N + TG_NT - 1) / TG_NT;
  p.m_tiles = (M + TG_BM - 1) / TG_BM;
  p.kb = K / TG_BK;
  p.U1 = (long long)p.n_tiles * p.kb;
  p.grid1 = (int)(p.U1 < TG_GRID ? p.U1 : TG_GRID);
  return p;
}

}  // namespace dfl

using namespace dfl;

extern "C" size_t dfl_gemm_workspace_bytes(int M, int N, int K, int epilogue) {
  (void)epilogue;
  if (M <= 0 || N <= 0 || K <= 0 || K % TG_BK) return 0;
  TgPlan p = tg_plan(M, N, K);
  return TG_COUNTER_BYTES + (size_t)p.m_tiles * p.grid1 * 2 * TG_BM * TG_NT * sizeof(float);
}

extern "C" int dfl_gemm_argmax_tiles(int N) { return (N + TG_NT - 1) / TG_NT; }

extern "C" int dfl_gemm_bf16(const void* x, int64_t ldx, const void* w, int M, int N, int K, int epilogue,
                             const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                             void* argmax_partials, const void* norm_w, const float* sumsq_in, int n_parts,
                             float eps, float* sumsq_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (M == 0) return DFL_OK;
  if (!x || !w || M < 0 || N <= 0 || K <= 0) {
    set_error("dfl_gemm_bf16: null pointer or bad shape M=%d N=%d K=%d", M, N, K);
    return DFL_ERR_INVALID;
  }
  if (K % TG_BK || N % 8 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15)) {
    set_error("dfl_gemm_bf16: needs K %% 128 == 0, N %% 8 == 0, 16-byte aligned x/w, ldx %% 8 == 0 (K=%d N=%d ldx=%lld)",
              K, N, (long long)ldx);
    return DFL_ERR_UNSUPPORTED;
  }
  if (epilogue == DFL_EPI_ARGMAX) {
    if (!argmax_partials) { set_error("dfl_gemm_bf16: argmax epilogue needs argmax_partials"); return DFL_ERR_INVALID; }
  } else if (!y || ldy % 8 || (y2 && ldy2 % 8) || (reinterpret_cast<uintptr_t>(y) & 15)) {
    set_error("dfl_gemm_bf16: y must be non-null, 16-byte aligned, ldy %% 8 == 0");
    return DFL_ERR_INVALID;
  }
  if (epilogue == DFL_EPI_RESIDUAL && (!residual || ldr % 8)) {
    set_error("dfl_gemm_bf16: residual epilogue needs a residual pointer with ldr %% 8 == 0");
    return DFL_ERR_INVALID;
  }
  if (epilogue == DFL_EPI_SILU_MUL && N % TG_NT) {
    set_error("dfl_gemm_bf16: silu-mul epilogue needs N %% 64 == 0 (packed gate/up), N=%d", N);
    return DFL_ERR_UNSUPPORTED;
  }
  if (norm_w && (!sumsq_in || n_parts <= 0 || K > TG_NORM_MAX_K)) {
    set_error("dfl_gemm_bf16: the fused RMSNorm prologue needs sumsq_in partials and K <= %d", TG_NORM_MAX_K);
    return DFL_ERR_INVALID;
  }
  TgPlan p = tg_plan(M, N, K);
  if ((size_t)p.m_tiles * p.n_tiles > (size_t)TG_MAX_COUNTERS) {
    set_error("dfl_gemm_bf16: too many output tiles (%d x %d)", p.m_tiles, p.n_tiles);
    return DFL_ERR_UNSUPPORTED;
  }
  const size_t need = dfl_gemm_workspace_bytes(M, N, K, epilogue);
  if (!workspace || workspace_bytes < need) {
    set_error("dfl_gemm_bf16: workspace too small (%zu < %zu bytes)", workspace_bytes, need);
    return DFL_ERR_WORKSPACE;
  }
  const CUtensorMap* wm = tensor_map_2d_bf16(w, N, K, K, TG_NT, 64);
  if (!wm) return DFL_ERR_CUDA;
  const CUtensorMap* xm = tensor_map_2d_bf16(x, M, K, ldx, TG_BM, 64);
  if (!xm) return DFL_ERR_CUDA;

  TgArgs a;
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.y2 = static_cast<__nv_bfloat16*>(y2);
  a.ldy2 = ldy2;
  a.argmax = static_cast<float2*>(argmax_partials);
  a.counters = static_cast<int*>(workspace);
  a.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + TG_COUNTER_BYTES);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.sumsq_in = sumsq_in;
  a.n_parts = n_parts;
  a.eps = eps;
  a.sumsq_out = sumsq_out;
  a.err = device_error_word();
  a.M = M;
  a.N = N;
  a.K = K;
  a.n_tiles = p.n_tiles;
  a.kb = p.kb;
  a.U1 = p.U1;
  a.grid1 = p.grid1;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid1 * p.m_tiles);
  cfg.blockDim = dim3(TG_THREADS);
  cfg.dynamicSmemBytes = TG_SMEM_BASE + (norm_w ? (size_t)K * 2 : 0);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err;
  switch (epilogue) {
#define DFL_LAUNCH(E)                                                                                      \
  case E: {                                                                                                \
    static bool init = false;                                                                              \
    if (!init) {                                                                                           \
      cudaFuncSetAttribute(gemm_tma_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,                \
                           TG_SMEM_BASE + TG_NORM_MAX_K * 2);                                              \
      init = true;                                                                                         \
    }                                                                                                      \
    err = cudaLaunchKernelEx(&cfg, gemm_tma_kernel<E>, *wm, *xm, a);                                       \
    break;                                                                                                 \
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

extern "C" int dfl_device_error(int* code, int clear, void* stream) {
  if (!code) return DFL_ERR_INVALID;
  cudaError_t e = cudaMemcpyFromSymbolAsync(code, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                            as_stream(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, as_stream(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  }
  if (e != cudaSuccess) {
    set_error("dfl_device_error: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}
