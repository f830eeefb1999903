// Persistent weight-streaming GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   Y[M, N] = Xn[M, K] . W[N, K]^T   (fp32 accumulate in TMEM) + fused epilogue
//   Xn      = X, or RMSNorm(X) with weight norm_w when the prologue is enabled
//
// Replaces the nn.Linear (and the RMSNorm feeding it) of the verify / draft
// forward: mlx-lm qwen3 Attention / MLP projections driven from
// adapters.py:611-631, DFlashAttention q/k/v/o (draft.py:75-98, 118-159), the
// draft fc + hidden_norm (draft.py:196-201, 217) and lm_head_logits /
// lm_head_argmax (adapters.py:264-271, 606-609; the argmax of runtime.py:22-29).
//
// B200 design
//  * Swap-AB: a 128-row tile of W is the MMA's M side (A operand, K-major,
//    128-byte swizzle) and the 16 tokens of X are its N side, so one
//    tcgen05.mma.cta_group::1.kind::f16 M=128 N=16 K=16 covers 128 outputs of all
//    16 rows; the accumulator lives in TMEM (2 buffers x 16 columns).
//  * W lives in HBM pre-tiled: every (128-row, 64-k) unit is one contiguous 16 KB
//    block already in the 128-byte-swizzle shared-memory image (dfl_pack_weight_bf16),
//    units ordered tile-major then k, so each CTA streams ONE contiguous byte range
//    with 1-D bulk copies.
//  * Warp roles: warp 0 = producer (1-D bulk copies of W with an evict-first L2
//    hint, 2-D TMA tile loads of X, evict-last), warp 1 = TMEM allocator + single-thread MMA issuer
//    (tcgen05.commit releases each shared-memory stage back to the producer),
//    warps 2-5 = epilogue (tcgen05.ld 32x32b: each thread owns one output column
//    for the 16 rows) and, when the RMSNorm is fused, the per-stage rescale of X.
//  * Persistent: two CTAs per SM per 16-row tile of X (grid 296); every CTA gets
//    an equal contiguous range of (128-row, 64-k) work units, so the SMs stream
//    equal shares of W and there is no tail wave. ~70 KB of shared memory per CTA lets
//    the next GEMM's CTA co-reside and stream its first weight stages before
//    griddepcontrol.wait (programmatic dependent launch).
//  * A tile cut by range boundaries is reduced by the last-arriving CTA in fixed
//    segment order; split points depend on N and K only, so every row is computed
//    with the same reduction order whatever M is (spec rows == plain-decode rows).
//  * Every mbarrier wait is bounded: on expiry the kernel records an error code in
//    the library's device error word and falls through to its teardown.
#include "tma_util.cuh"
#include "tcgen05.cuh"
#include "rope.cuh"

#include <cstring>
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


constexpr int TC_NT = 128;  // W rows per tile (MMA M)
constexpr int TC_BK = 64;   // k per stage (one 128-byte swizzle row)
constexpr int TC_BM = 16;   // tokens per tile (MMA N)
#ifndef DFL_TC_STAGES
#define DFL_TC_STAGES 3
#endif
constexpr int TC_STAGES = DFL_TC_STAGES;
#ifndef DFL_TC_GRID
#define DFL_TC_GRID 296
#endif
// Work split: two streaming CTAs per SM (148 SMs) plus room for the next kernel's
// prologue; one CTA alone cannot keep enough bulk copies in flight. Fixed: part of
// the reduction order.
constexpr int TC_GRID = DFL_TC_GRID;
constexpr int TC_THREADS = 192;
constexpr int TC_EPI_WARP0 = 2;
constexpr int TC_W_BYTES = TC_NT * TC_BK * 2;  // 16 KB
constexpr int TC_X_BYTES = TC_BM * TC_BK * 2;  // 2 KB
constexpr int TC_OFF_X = TC_STAGES * TC_W_BYTES;
constexpr int TC_OFF_XCHG = TC_OFF_X + TC_STAGES * TC_X_BYTES;
constexpr int TC_OFF_BAR = TC_OFF_XCHG + TC_NT * TC_BM * 4;  // exchange / cluster-reduction tile (8 KB)
constexpr int TC_NBAR = 3 * TC_STAGES + 4;
constexpr int TC_OFF_TMEM = TC_OFF_BAR + TC_NBAR * 8;
constexpr int TC_OFF_NORM = (TC_OFF_TMEM + 16 + 127) & ~127;
constexpr int TC_SMEM_BASE = TC_OFF_NORM + 1024;  // + 1024-byte alignment slack
constexpr int TC_NORM_MAX_K = 8192;
// Independent TMEM accumulators per tile: the four K=16 MMAs of a stage go to
// different accumulators so that consecutive MMAs do not wait on each other; the
// epilogue sums them in a fixed order.
#ifndef DFL_TC_NACC
#define DFL_TC_NACC 4
#endif
constexpr int TC_NACC = DFL_TC_NACC;
#ifndef DFL_TC_PLANES
#define DFL_TC_PLANES 1
#endif
constexpr int TC_PLANES = DFL_TC_PLANES;
#ifndef DFL_TC_MINB
#define DFL_TC_MINB 3
#endif
constexpr int TC_PB = 2;  // partial tiles loaded per round by a split-tile reducer
#ifndef DFL_TC_SMAX
#define DFL_TC_SMAX 8
#endif
constexpr int TC_TMEM_COLS = 2 * TC_NACC * TC_BM <= 32 ? 32 : (2 * TC_NACC * TC_BM <= 64 ? 64 : 128);
constexpr int TC_MAX_COUNTERS = 1 << 17;
constexpr size_t TC_COUNTER_BYTES = (size_t)TC_MAX_COUNTERS * sizeof(int);
constexpr int TC_PART_FLOATS = TC_BM * TC_NT;  // one partial tile

// tcgen05 instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major,
// N = 16 (bits 17-22: N >> 3), M = 128 (bits 24-28: M >> 4).
constexpr uint32_t TC_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_BM >> 3) << 17) |
                              ((uint32_t)(TC_NT >> 4) << 24);

constexpr int TC_KV_LAYERS_MAX = 16;  // layers one fused context K/V projection may append

struct TcArgs {
  const unsigned char* wt;  // pre-tiled weights: unit u at wt + u * TC_W_BYTES
  const __nv_bfloat16* res;
  long long ldr;
  __nv_bfloat16* y;
  long long ldy;
  __nv_bfloat16* y2;
  long long ldy2;
  float2* argmax;  // [M][N/32]
  float* partial;  // [m_tiles][grid1][2][128 cols][16 rows]
  int* counters;   // [m_tiles * n_tiles]
  const __nv_bfloat16* norm_w;
  const float* sumsq_in;  // [M][n_parts] (n_parts = K/32)
  int n_parts;
  float eps;
  float* sumsq_out;  // [M][N/32]
  int* err;
  int n_groups;  // N / 32: row stride of sumsq_out and argmax
  int M, N, K, n_tiles, kb;
  long long U1;
  int grid1;
  // fused q/k head norm + RoPE + KV append after the QKV projection (cluster split-K form,
  // head_dim 128 = one column tile per head, M <= 16): rope_on selects it
  int rope_on;
  QkvArgs rope;
  // several layers' context-row K/V in one projection (rope.Hq = 0): 2 Hkv column tiles per
  // layer, layer l's k_norm weight at rope_k_norm[l]; 0 = one layer
  int rope_layer_heads;
  const __nv_bfloat16* rope_k_norm[TC_KV_LAYERS_MAX];
};

// tcgen05 helpers (descriptors, MMA issue, commit, fences, TMEM loads): tcgen05.cuh

// Sum of the TC_NACC accumulators of one buffer, in a fixed order.
__device__ __forceinline__ void tc_ld_acc(uint32_t taddr, float* v) {
  tc_ld16(taddr, v);
#pragma unroll
  for (int k = 1; k < TC_NACC; ++k) {
    float w[16];
    tc_ld16(taddr + (uint32_t)(k * TC_BM), w);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += w[i];
  }
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

__device__ __forceinline__ int tc_unit_owner(long long u, long long U, int G) {
  return (int)(((u + 1) * G + U - 1) / U) - 1;
}

// Epilogue from registers: this thread owns column n (tile column c = q*32 + lane)
// for the 16 rows m0 .. m0 + 15; q is the thread's TMEM lane quadrant.
template <int EPI>
__device__ __forceinline__ void tc_epilogue(const TcArgs& a, float* v, int m0, int nt, int q, int lane,
                                            float* xchg, const float* rpre = nullptr) {
  const int c = q * 32 + lane;
  const int n = nt * TC_NT + c;
  if constexpr (EPI == DFL_EPI_STORE_F32) {
    float* yf = reinterpret_cast<float*>(a.y);
#pragma unroll
    for (int t = 0; t < TC_BM; ++t)
      if (n < a.N && m0 + t < a.M) yf[(long long)(m0 + t) * a.ldy + n] = v[t];
  } else if constexpr (EPI == DFL_EPI_STORE || EPI == DFL_EPI_RESIDUAL) {
    const bool col_ok = n < a.N;
    if constexpr (EPI == DFL_EPI_RESIDUAL) {
      // gather all 16 residual values before the first store: y may alias the residual
      // (in-place update), so interleaved loads and stores would serialise 16 L2 round trips
      float r[TC_BM];
      if (rpre) {
#pragma unroll
        for (int t = 0; t < TC_BM; ++t) r[t] = rpre[t];
      } else {
#pragma unroll
        for (int t = 0; t < TC_BM; ++t)
          r[t] = (col_ok && m0 + t < a.M)
                     ? __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(a.res) +
                                                        (long long)(m0 + t) * a.ldr + n) << 16)
                     : 0.f;
      }
#pragma unroll
      for (int t = 0; t < TC_BM; ++t) v[t] = r[t] + round_bf16(v[t]);
    }
#pragma unroll
    for (int t = 0; t < TC_BM; ++t) {
      const int m = m0 + t;
      float ss = 0.f;
      if (col_ok && m < a.M) {
        const __nv_bfloat16 o = f2bf(v[t]);
        a.y[(long long)m * a.ldy + n] = o;
        if (a.y2) a.y2[(long long)m * a.ldy2 + n] = o;
        const float qv = bf2f(o);
        ss = qv * qv;
      }
      if (a.sumsq_out) {
        ss = warp_sum(ss);
        if (lane == 0 && m < a.M && nt * 4 + q < a.n_groups) a.sumsq_out[(long long)m * a.n_groups + nt * 4 + q] = ss;
      }
    }
  } else if constexpr (EPI == DFL_EPI_ARGMAX) {
#pragma unroll
    for (int t = 0; t < TC_BM; ++t) {
      float best = n < a.N ? round_bf16(v[t]) : -INFINITY;
      int bidx = n < a.N ? n : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (ob > best || (ob == best && oi < bidx)) { best = ob; bidx = oi; }
      }
      const int m = m0 + t;
      if (lane == 0 && m < a.M && nt * 4 + q < a.n_groups)
        a.argmax[(long long)m * a.n_groups + nt * 4 + q] = make_float2(best, __int_as_float(bidx));
    }
  } else if constexpr (EPI == DFL_EPI_SILU_MUL) {
    // packed per 64 W rows as [32 gate | 32 up]: quadrants 0/2 hold gate rows, 1/3 the matching up rows
    const int g = q >> 1;
    if (q & 1) {
#pragma unroll
      for (int t = 0; t < TC_BM; ++t) xchg[(g * TC_BM + t) * 32 + lane] = v[t];
    }
    epi_sync();
    if (!(q & 1)) {
      const int on = nt * 64 + g * 32 + lane;
      if (nt * TC_NT + c < a.N) {
#pragma unroll
        for (int t = 0; t < TC_BM; ++t) {
          const int m = m0 + t;
          if (m < a.M) {
            const float gt = round_bf16(v[t]);
            const float up = round_bf16(xchg[(g * TC_BM + t) * 32 + lane]);
            const float act = round_bf16(gt / (1.f + __expf(-gt)));
            a.y[(long long)m * a.ldy + on] = f2bf(act * up);
          }
        }
      }
    }
    epi_sync();
  }
}

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, DFL_TC_MINB)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap, TcArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_OFF_BAR);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* xready = empty + TC_STAGES;
  uint64_t* accf = xready + TC_STAGES;  // [2]
  uint64_t* acce = accf + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TC_OFF_TMEM);
  float* xchg = reinterpret_cast<float*>(smem + TC_OFF_XCHG);
  __nv_bfloat16* s_nw = reinterpret_cast<__nv_bfloat16*>(smem + TC_OFF_NORM);
  __shared__ float s_inv[TC_BM];
  __shared__ int s_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x / a.grid1;
  const int c = blockIdx.x % a.grid1;
  const long long u0 = (long long)c * a.U1 / a.grid1;
  const long long u1 = (long long)(c + 1) * a.U1 / a.grid1;
  const int n_units = (int)(u1 - u0);
  const bool norm = a.norm_w != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&xready[s], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "n"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // TC_PLANES lanes each copy one slice of every weight stage (parallel bulk copies)
    constexpr unsigned PMASK = (1u << TC_PLANES) - 1u;
    constexpr uint32_t SLICE = TC_W_BYTES / TC_PLANES;
    if (lane < TC_PLANES && n_units > 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const int pre = n_units < TC_STAGES ? n_units : TC_STAGES;
      for (int i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        if (lane == 0) mbar_expect_tx(&full[i], TC_W_BYTES + TC_X_BYTES);
        __syncwarp(PMASK);
        bulk_load(smem + i * TC_W_BYTES + lane * SLICE, a.wt + u * TC_W_BYTES + lane * SLICE, SLICE, &full[i], pol_w);
      }
      grid_dependency_wait();  // X is produced by the previous kernel
      if (lane == 0) {
        for (int i = 0; i < pre; ++i)
          tma_load_2d(&xmap, &full[i], smem + TC_OFF_X + i * TC_X_BYTES, (int)((u0 + i) % a.kb) * TC_BK, mt * TC_BM,
                      pol_x);
      }
      int issued = pre;
      for (int i = pre; i < n_units; ++i) {
        const int s = i % TC_STAGES;
        if (!mbar_wait(&empty[s], ((i / TC_STAGES) & 1) ^ 1, 201, a.err)) break;
        const long long u = u0 + i;
        if (lane == 0) mbar_expect_tx(&full[s], TC_W_BYTES + TC_X_BYTES);
        __syncwarp(PMASK);
        bulk_load(smem + s * TC_W_BYTES + lane * SLICE, a.wt + u * TC_W_BYTES + lane * SLICE, SLICE, &full[s], pol_w);
        if (lane == 0)
          tma_load_2d(&xmap, &full[s], smem + TC_OFF_X + s * TC_X_BYTES, (int)(u % a.kb) * TC_BK, mt * TC_BM, pol_x);
        issued = i + 1;
      }
      if (issued < n_units && lane == 0) {
        // gave up: let the copies already in flight land before the CTA exits
        for (int i = issued > TC_STAGES ? issued - TC_STAGES : 0; i < issued; ++i)
          mbar_wait(&full[i % TC_STAGES], (i / TC_STAGES) & 1, 209, a.err);
      }
    }
    __syncwarp();  // lanes 1-31 wait for the producing lane before the teardown barrier
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_units > 0) {
      const uint32_t w0 = smem_u32(smem), x0 = smem_u32(smem + TC_OFF_X);
      int seg = -1;
      for (int i = 0; i < n_units; ++i) {
        const long long u = u0 + i;
        const int j = (int)(u % a.kb);
        const int s = i % TC_STAGES;
        const bool first = (i == 0) || (j == 0);
        if (first) {
          ++seg;
          if (!mbar_wait(&acce[seg & 1], ((seg >> 1) & 1) ^ 1, 202, a.err)) break;
          tc_fence_after();
        }
        if (!mbar_wait(norm ? &xready[s] : &full[s], (i / TC_STAGES) & 1, 203, a.err)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)((seg & 1) * TC_NACC * TC_BM);
        const uint64_t ad = sw128_desc(w0 + s * TC_W_BYTES);
        const uint64_t bd = sw128_desc(x0 + s * TC_X_BYTES);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 16; ++kk)  // +32 bytes along K per MMA: +2 in the start-address field
          tc_mma(d + (uint32_t)((kk % TC_NACC) * TC_BM), ad + 2 * kk, bd + 2 * kk, TC_IDESC,
                 (first && kk < TC_NACC) ? 0u : 1u);
        tc_commit(&empty[s]);
        if (j == a.kb - 1 || i == n_units - 1) tc_commit(&accf[seg & 1]);
      }
    }
    __syncwarp();  // the whole warp reaches the teardown (and the .sync.aligned dealloc) together
  } else {
    // ---------------- epilogue warps (and the fused RMSNorm rescale) ----------------
    const int ew = warp - TC_EPI_WARP0;  // 0..3
    const int et = threadIdx.x - 32 * TC_EPI_WARP0;  // 0..127
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    if (norm)
      for (int k = et * 8; k < a.K; k += 128 * 8)
        *reinterpret_cast<uint4*>(s_nw + k) = *reinterpret_cast<const uint4*>(a.norm_w + k);
    grid_dependency_wait();
    if (norm) {
      if (et < TC_BM) {
        const int m = mt * TC_BM + et;
        float ss = 0.f;
        if (m < a.M)
          for (int p = 0; p < a.n_parts; ++p) ss += a.sumsq_in[(long long)m * a.n_parts + p];
        s_inv[et] = rsqrtf(ss / (float)a.K + a.eps);
      }
      epi_sync();
    }
    int seg = -1;
    for (int i = 0; i < n_units; ++i) {
      const long long u = u0 + i;
      const int nt = (int)(u / a.kb), j = (int)(u % a.kb);
      const int s = i % TC_STAGES;
      if (i == 0 || j == 0) ++seg;
      if (norm) {
        if (!mbar_wait(&full[s], (i / TC_STAGES) & 1, 204, a.err)) break;
        // rescale this thread's 16-byte chunk of the X stage: xn = bf16(w * x * inv_rms)
        const int row = et >> 3, cc = et & 7;
        __nv_bfloat16* p =
            reinterpret_cast<__nv_bfloat16*>(smem + TC_OFF_X + s * TC_X_BYTES) + row * 64 + ((cc ^ (row & 7)) << 3);
        uint4 xv = *reinterpret_cast<uint4*>(p);
        const uint4 wv = *reinterpret_cast<const uint4*>(s_nw + j * TC_BK + cc * 8);
        __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
        const float inv = s_inv[row];
#pragma unroll
        for (int e = 0; e < 8; ++e) xe[e] = f2bf(bf2f(we[e]) * (bf2f(xe[e]) * inv));
        *reinterpret_cast<uint4*>(p) = xv;
        fence_proxy_async_smem();  // generic writes -> visible to the tensor core's async-proxy reads
        mbar_arrive(&xready[s]);
      }
      const bool seg_end = (j == a.kb - 1) || (i == n_units - 1);
      if (!seg_end) continue;
      if (!mbar_wait(&accf[seg & 1], (seg >> 1) & 1, 205, a.err)) break;
      tc_fence_after();
      float v[TC_BM];
      tc_ld_acc(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((seg & 1) * TC_NACC * TC_BM), v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[seg & 1]);

      const long long tu0 = (long long)nt * a.kb, tu1 = tu0 + a.kb - 1;
      const int c_first = tc_unit_owner(tu0, a.U1, a.grid1), c_last = tc_unit_owner(tu1, a.U1, a.grid1);
      bool do_epi = true;
      const int col = q * 32 + lane;
      if (c_first != c_last) {
        const int tile_id = mt * a.n_tiles + nt;
        const int slot = (nt == (int)(u0 / a.kb)) ? 0 : 1;
        float4* mine = reinterpret_cast<float4*>(a.partial + (((long long)mt * a.grid1 + c) * 2 + slot) * TC_PART_FLOATS +
                                                 col * TC_BM);
#pragma unroll
        for (int t4 = 0; t4 < TC_BM / 4; ++t4) mine[t4] = make_float4(v[4 * t4], v[4 * t4 + 1], v[4 * t4 + 2], v[4 * t4 + 3]);
        asm volatile("fence.acq_rel.gpu;\n" ::: "memory");  // publish this segment's partial
        epi_sync();
        if (et == 0) {
          int prev;
          asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;\n" : "=r"(prev) : "l"(a.counters + tile_id) : "memory");
          s_flag = (prev == c_last - c_first);
        }
        epi_sync();
        do_epi = s_flag != 0;
        if (do_epi) {
          asm volatile("fence.acq_rel.gpu;\n" ::: "memory");  // see every segment's partial
#pragma unroll
          for (int t = 0; t < TC_BM; ++t) v[t] = 0.f;
          // TC_PB segments' partials in flight per round, summed in segment order
          for (int cs0 = c_first; cs0 <= c_last; cs0 += TC_PB) {
            float4 pb[TC_PB][TC_BM / 4];
#pragma unroll
            for (int k = 0; k < TC_PB; ++k) {
              const int cs = cs0 + k;
              if (cs <= c_last) {
                const long long cs_u0 = (long long)cs * a.U1 / a.grid1;
                const int sl = (nt == (int)(cs_u0 / a.kb)) ? 0 : 1;
                const float4* src = reinterpret_cast<const float4*>(
                    a.partial + (((long long)mt * a.grid1 + cs) * 2 + sl) * TC_PART_FLOATS + col * TC_BM);
#pragma unroll
                for (int t4 = 0; t4 < TC_BM / 4; ++t4) pb[k][t4] = __ldcg(src + t4);
              }
            }
#pragma unroll
            for (int k = 0; k < TC_PB; ++k) {
              if (cs0 + k <= c_last) {
#pragma unroll
                for (int t4 = 0; t4 < TC_BM / 4; ++t4) {
                  v[4 * t4] += pb[k][t4].x;
                  v[4 * t4 + 1] += pb[k][t4].y;
                  v[4 * t4 + 2] += pb[k][t4].z;
                  v[4 * t4 + 3] += pb[k][t4].w;
                }
              }
            }
          }
          if (et == 0) {
            a.counters[tile_id] = 0;  // ready for the next launch / graph replay
          }
        }
        epi_sync();  // s_flag is rewritten by the next segment
      }
      if (do_epi) tc_epilogue<EPI>(a, v, mt * TC_BM, nt, q, lane, xchg);
      (void)ew;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "n"(TC_TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// Cluster split-K variant for GEMMs with few 128-row tiles (N / 128 < DFL_TC_CSK_TILES, the stream-K grid):
// a thread-block cluster of S CTAs (S <= 8) owns one tile, CTA rank r streams the
// fixed k-range [r*kb/S, (r+1)*kb/S), and the S partial tiles are reduced through
// distributed shared memory in rank order (no global scratch, no atomics). Each
// 32-column group of the tile is finished by one owner rank: every other rank pushes
// its fp32 partial columns into the owner's receive slots with st.async (completing on
// an mbarrier in the owner), so no rank waits on a remote load; the owner sums the
// ranks in rank order. Residual columns are loaded by the owner while the weights
// stream. (Pulling the partials with ld.shared::cluster after a cluster barrier cost
// 4-9 us per launch while other clusters' weight streams held the SM-to-SM network.)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;\n" ::: "memory");
}
// 16-byte store into another CTA's shared memory that completes on an mbarrier there
__device__ __forceinline__ void st_async_v4(uint32_t addr, float x, float y, float z, float w, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];\n" ::"r"(addr),
               "f"(x), "f"(y), "f"(z), "f"(w), "r"(bar)
               : "memory");
}
constexpr int TC_CSK_SLOT_BYTES = 32 * TC_BM * 4;  // one rank's partial of a 32-column group
// Cluster-kernel shared memory: ring | X | barriers | TMEM slot | norm weights (K*2 when
// fused) | receive slots (when they fit beside three co-resident CTAs; otherwise the
// pushes land in the idle ring).
constexpr int CSK_OFF_BAR = TC_OFF_X + TC_STAGES * TC_X_BYTES;
constexpr int CSK_OFF_TMEM = CSK_OFF_BAR + TC_NBAR * 8;
constexpr int CSK_OFF_NORM = (CSK_OFF_TMEM + 16 + 127) & ~127;
constexpr int CSK_SMEM_PER_SM = 228 * 1024, CSK_RESERVED_PER_CTA = 1024;

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, DFL_TC_MINB)
    gemm_csk_kernel(const __grid_constant__ CUtensorMap xmap, TcArgs a, int S, int recv_off) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + CSK_OFF_BAR);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* xready = empty + TC_STAGES;
  uint64_t* accf = xready + TC_STAGES;
  uint64_t* recv = accf + 1;  // [2]: pushes of the column groups this rank owns
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + CSK_OFF_TMEM);
  __nv_bfloat16* s_nw = reinterpret_cast<__nv_bfloat16*>(smem + CSK_OFF_NORM);
  unsigned char* rbuf = smem + recv_off;  // receive slots (offset 0: the weight ring)
  const bool dedicated = recv_off != 0;
  __shared__ float s_inv[TC_BM];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x;  // rank in the cluster (cluster dims = (S, 1, 1), gridDim.x == S)
  const int nt = blockIdx.y, mt = blockIdx.z;
  const int j0 = r * a.kb / S, j1 = (r + 1) * a.kb / S;
  const int n_units = j1 - j0;
  const bool norm = a.norm_w != nullptr;
  const int cta_lin = r + S * (nt + a.n_tiles * mt);
  (void)cta_lin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&xready[s], 128);
    }
    mbar_init(&accf[0], 1);
    // owned units: column groups q (or SILU gate/up pairs) with unit % S == r
    const int U = EPI == DFL_EPI_SILU_MUL ? 2 : 4;
    const int per = EPI == DFL_EPI_SILU_MUL ? 2 * S : S - 1;
    for (int u = r; u < U && per > 0; u += S) mbar_init(&recv[u / S], 1);
    fence_barrier_init();
    for (int u = r; u < U && per > 0; u += S) mbar_expect_tx(&recv[u / S], (uint32_t)(per * TC_CSK_SLOT_BYTES));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "n"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_launch_dependents();
  // dedicated receive slots: the only cluster-wide precondition of a push is that the
  // owner's barriers are initialised (arrive now, wait just before pushing)
  if (dedicated) cluster_arrive_relaxed();  // the barrier inits were published by fence.mbarrier_init
  // residual columns of the warps that finish a column group: loaded while the weights
  // stream (a load issued after the reduction waits behind the other clusters' streams)
  float rres[TC_BM], v[TC_BM];
#pragma unroll
  for (int t = 0; t < TC_BM; ++t) rres[t] = v[t] = 0.f;

  if (warp == 0) {
    if (lane == 0 && n_units > 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const long long ubase = (long long)nt * a.kb + j0;
      const int pre = n_units < TC_STAGES ? n_units : TC_STAGES;
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], TC_W_BYTES + TC_X_BYTES);
        bulk_load(smem + i * TC_W_BYTES, a.wt + (ubase + i) * TC_W_BYTES, TC_W_BYTES, &full[i], pol_w);
      }
      grid_dependency_wait();  // X is produced by the previous kernel
      for (int i = 0; i < pre; ++i)
        tma_load_2d(&xmap, &full[i], smem + TC_OFF_X + i * TC_X_BYTES, (j0 + i) * TC_BK, mt * TC_BM, pol_x);
      int issued = pre;
      for (int i = pre; i < n_units; ++i) {
        const int s = i % TC_STAGES;
        if (!mbar_wait(&empty[s], ((i / TC_STAGES) & 1) ^ 1, 301, a.err)) break;
        mbar_expect_tx(&full[s], TC_W_BYTES + TC_X_BYTES);
        bulk_load(smem + s * TC_W_BYTES, a.wt + (ubase + i) * TC_W_BYTES, TC_W_BYTES, &full[s], pol_w);
        tma_load_2d(&xmap, &full[s], smem + TC_OFF_X + s * TC_X_BYTES, (j0 + i) * TC_BK, mt * TC_BM, pol_x);
        issued = i + 1;
      }
      if (issued < n_units)
        for (int i = issued > TC_STAGES ? issued - TC_STAGES : 0; i < issued; ++i)
          mbar_wait(&full[i % TC_STAGES], (i / TC_STAGES) & 1, 309, a.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && n_units > 0) {
      const uint32_t w0 = smem_u32(smem), x0 = smem_u32(smem + TC_OFF_X);
      for (int i = 0; i < n_units; ++i) {
        const int s = i % TC_STAGES;
        if (!mbar_wait(norm ? &xready[s] : &full[s], (i / TC_STAGES) & 1, 303, a.err)) break;
        tc_fence_after();
        const uint64_t ad = sw128_desc(w0 + s * TC_W_BYTES);
        const uint64_t bd = sw128_desc(x0 + s * TC_X_BYTES);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 16; ++kk)
          tc_mma(tmem + (uint32_t)((kk % TC_NACC) * TC_BM), ad + 2 * kk, bd + 2 * kk, TC_IDESC,
                 (i == 0 && kk < TC_NACC) ? 0u : 1u);
        tc_commit(&empty[s]);
      }
      tc_commit(&accf[0]);
    }
    __syncwarp();
  } else {
    const int et = threadIdx.x - 32 * TC_EPI_WARP0;
    const int q = warp & 3;
    if (norm)
      for (int k = et * 8; k < a.K; k += 128 * 8)
        *reinterpret_cast<uint4*>(s_nw + k) = *reinterpret_cast<const uint4*>(a.norm_w + k);
    grid_dependency_wait();
    if constexpr (EPI == DFL_EPI_RESIDUAL) {
      const int n = nt * TC_NT + q * 32 + lane;
      if ((q % S) == r && n < a.N) {
#pragma unroll
        for (int t = 0; t < TC_BM; ++t)
          if (mt * TC_BM + t < a.M) rres[t] = bf2f(a.res[(long long)(mt * TC_BM + t) * a.ldr + n]);
      }
    }
    if (norm) {
      if (et < TC_BM) {
        const int m = mt * TC_BM + et;
        float ss = 0.f;
        if (m < a.M)
          for (int p = 0; p < a.n_parts; ++p) ss += a.sumsq_in[(long long)m * a.n_parts + p];
        s_inv[et] = rsqrtf(ss / (float)a.K + a.eps);
      }
      epi_sync();
      for (int i = 0; i < n_units; ++i) {
        const int s = i % TC_STAGES;
        if (!mbar_wait(&full[s], (i / TC_STAGES) & 1, 304, a.err)) break;
        const int j = j0 + i;
        const int row = et >> 3, cc = et & 7;
        __nv_bfloat16* p =
            reinterpret_cast<__nv_bfloat16*>(smem + TC_OFF_X + s * TC_X_BYTES) + row * 64 + ((cc ^ (row & 7)) << 3);
        uint4 xv = *reinterpret_cast<uint4*>(p);
        const uint4 wv = *reinterpret_cast<const uint4*>(s_nw + j * TC_BK + cc * 8);
        __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
        const float inv = s_inv[row];
#pragma unroll
        for (int e = 0; e < 8; ++e) xe[e] = f2bf(bf2f(we[e]) * (bf2f(xe[e]) * inv));
        *reinterpret_cast<uint4*>(p) = xv;
        fence_proxy_async_smem();
        mbar_arrive(&xready[s]);
      }
    }
    if (n_units > 0 && mbar_wait(&accf[0], 0, 305, a.err)) {
      tc_fence_after();
      tc_ld_acc(tmem + ((uint32_t)(q * 32) << 16), v);
      tc_fence_before();
    }
  }
  // Cluster reduction by push: every rank sends its partial column group to the group's
  // owner rank with st.async into the owner's receive slots, completing on an mbarrier
  // there; the owner sums the ranks in rank order. Slots in the weight ring need every
  // ring free first (each CTA's epilogue warps passed accf, so its MMAs are done).
  if (dedicated)
    cluster_wait();
  else
    cluster_sync_all();
  constexpr bool SILU = EPI == DFL_EPI_SILU_MUL;
  const int slots = SILU ? 2 * S : S - 1;  // per owned unit
  if (warp >= TC_EPI_WARP0) {
    const int q = warp & 3;
    const int u = SILU ? q >> 1 : q, gi = SILU ? q & 1 : 0;
    const int owner = u % S, js = u / S;
    if (SILU || owner != r) {
      const int slot = SILU ? 2 * r + gi : (r < owner ? r : r - 1);
      const uint32_t dst = cluster_map(smem_u32(rbuf + (js * slots + slot) * TC_CSK_SLOT_BYTES + lane * 64), owner);
      const uint32_t bar = cluster_map(smem_u32(&recv[js]), owner);
#pragma unroll
      for (int t4 = 0; t4 < TC_BM / 4; ++t4)
        st_async_v4(dst + t4 * 16, v[4 * t4], v[4 * t4 + 1], v[4 * t4 + 2], v[4 * t4 + 3], bar);
    }
  }
  cluster_arrive();  // phase 2: this CTA's pushes are issued
  if (warp >= TC_EPI_WARP0) {
    const int q = warp & 3;
    const int u = SILU ? q >> 1 : q;
    const int owner = u % S, js = u / S;
    if (owner == r && (!SILU || !(q & 1))) {
      if (slots > 0 && !mbar_wait(&recv[js], 0, 306, a.err)) {
        // gave up: the sums below read whatever arrived; the error word reports it
      }
      const float* base = reinterpret_cast<const float*>(rbuf + js * slots * TC_CSK_SLOT_BYTES) + lane * 16;
      if constexpr (SILU) {
        float gv[TC_BM], uv[TC_BM];
#pragma unroll
        for (int t = 0; t < TC_BM; ++t) gv[t] = uv[t] = 0.f;
        for (int rr = 0; rr < S; ++rr) {
          const float4* g4 = reinterpret_cast<const float4*>(base + (2 * rr) * (TC_CSK_SLOT_BYTES / 4));
          const float4* u4 = reinterpret_cast<const float4*>(base + (2 * rr + 1) * (TC_CSK_SLOT_BYTES / 4));
#pragma unroll
          for (int t4 = 0; t4 < TC_BM / 4; ++t4) {
            const float4 g = g4[t4], w = u4[t4];
            gv[4 * t4] += g.x; gv[4 * t4 + 1] += g.y; gv[4 * t4 + 2] += g.z; gv[4 * t4 + 3] += g.w;
            uv[4 * t4] += w.x; uv[4 * t4 + 1] += w.y; uv[4 * t4 + 2] += w.z; uv[4 * t4 + 3] += w.w;
          }
        }
        const int on = nt * 64 + u * 32 + lane;
        if (nt * TC_NT + q * 32 + lane < a.N) {
#pragma unroll
          for (int t = 0; t < TC_BM; ++t) {
            const int m = mt * TC_BM + t;
            if (m < a.M) {
              const float gt = round_bf16(gv[t]);
              const float up = round_bf16(uv[t]);
              const float act = round_bf16(gt / (1.f + __expf(-gt)));
              a.y[(long long)m * a.ldy + on] = f2bf(act * up);
            }
          }
        }
      } else {
        float acc[TC_BM];
#pragma unroll
        for (int t = 0; t < TC_BM; ++t) acc[t] = 0.f;
        for (int rr = 0; rr < S; ++rr) {  // rank order; this rank's own partial from registers
          if (rr == r) {
#pragma unroll
            for (int t = 0; t < TC_BM; ++t) acc[t] += v[t];
          } else {
            const float4* p4 =
                reinterpret_cast<const float4*>(base + (rr < r ? rr : rr - 1) * (TC_CSK_SLOT_BYTES / 4));
#pragma unroll
            for (int t4 = 0; t4 < TC_BM / 4; ++t4) {
              const float4 f = p4[t4];
              acc[4 * t4] += f.x; acc[4 * t4 + 1] += f.y; acc[4 * t4 + 2] += f.z; acc[4 * t4 + 3] += f.w;
            }
          }
        }
        tc_epilogue<EPI>(a, acc, mt * TC_BM, nt, q, lane, nullptr, rres);
      }
    }
  }
  cluster_wait();  // no CTA leaves while a push to it may be in flight
  if (EPI == DFL_EPI_STORE && a.rope_on) {
    // fused q/k head norm + RoPE + KV append: column tile nt is head nt. One more cluster
    // barrier makes every owner's stores of the tile visible to the whole cluster; the rows
    // are then spread over the ranks' warps (row m on rank m % S), each running
    // dfl_qkv_rope_append's arithmetic with the idle weight ring as its row buffer.
    cluster_arrive();
    cluster_wait();
    float* buf = reinterpret_cast<float*>(smem) + warp * 128;
    const int lh = a.rope_layer_heads;
    const int layer = lh ? nt / lh : 0, head = lh ? nt % lh : nt;
    const __nv_bfloat16* knl = lh ? a.rope_k_norm[layer] : nullptr;
    for (int m = r + S * warp; m < a.M; m += S * (TC_THREADS / 32)) qkv_rope_row(a.rope, m, head, lane, buf, layer, knl);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "n"(TC_TMEM_COLS));
  }
}

// Row-major W [N, K] -> tiled image: unit (tile t, k-block j) at ((t*kb)+j)*16 KB, row r
// (W row t*128+r, zero past N) holding 16-byte chunk c of k-block j at r*128 + ((c^(r&7))*16).
__global__ void pack_weight_kernel(const __nv_bfloat16* __restrict__ w, int N, int K,
                                   unsigned char* __restrict__ out, long long n_chunks) {
  const int kb = K / TC_BK;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_chunks; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i & 7);
    const long long rowchunk = i >> 3;  // global tiled row index within units
    const int r = (int)(rowchunk % TC_NT);
    const long long unit = rowchunk / TC_NT;
    const int j = (int)(unit % kb);
    const long long t = unit / kb;
    const long long n = t * TC_NT + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < N) v = *reinterpret_cast<const uint4*>(w + n * (long long)K + (long long)j * TC_BK + c * 8);
    *reinterpret_cast<uint4*>(out + unit * TC_W_BYTES + r * 128 + ((c ^ (r & 7)) << 4)) = v;
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

// ---------------------------------------------------------------------------
// Wide GEMM: the many-row form (batched verify, 64+ sequences x 16 rows).
//
// Same pre-tiled weight stream, instruction shape M = 128 weight rows x N = BN tokens
// (BN <= 256, a multiple of 16) and the same epilogues, but every output tile
// (128 weight rows x BN rows of X) is owned by one CTA that runs the whole K loop
// into one TMEM accumulator: there is no split-K, so a row's result depends on K
// order only (identical for any number of rows, any BN). Persistent: one CTA per
// SM walks the tiles with the row tiles of one weight strip adjacent, so the CTAs
// that read the same 16 KB weight unit run at the same time and share it in L2.
// 4-stage ring of (16 KB weight unit + BN x 64 X tile), double-buffered accumulator
// (2 x BN TMEM columns) so the epilogue of tile i overlaps the MMAs of tile i + 1.
// The RMSNorm prologue, when requested, runs as a separate row kernel into the
// workspace (xn = bf16(w * x * inv_rms), the fused prologue's formula).
// ---------------------------------------------------------------------------
constexpr int WG_BN_MAX = 256;
constexpr int WG_MAX_STAGES = 8;
constexpr int WG_RING_BYTES = 192 * 1024;  // weight + X stages; as many stages as fit (4 at BN 256)
constexpr int WG_EPI_LD = TC_NT + 4;  // fp32 row pitch of the epilogue transpose tile
constexpr int WG_OFF_EPI = WG_RING_BYTES;
constexpr int WG_OFF_BAR = WG_OFF_EPI + TC_BM * WG_EPI_LD * 4;
constexpr int WG_NBAR = 2 * WG_MAX_STAGES + 4;
constexpr int WG_OFF_TMEM = WG_OFF_BAR + WG_NBAR * 8;
constexpr int WG_SMEM = WG_OFF_TMEM + 16 + 1024;

struct WgArgs {
  TcArgs t;
  float* part;  // split > 1: fp32 partials [split][M][N] (reduced in order by wide_split_reduce_kernel)
  int split;    // K ranges per tile (1: the tile's epilogue runs here)
  int stages;   // ring depth: W stages at 0, X stages after them
  int bn;       // tokens per tile
  int m_tiles;  // row tiles of X
  int tiles;    // n_tiles * m_tiles
};

// Wide-kernel epilogue for 16 rows m0 .. m0 + 15 of one 128-column tile. The TMEM
// layout gives thread c the column c for all 16 rows; the values are transposed
// through shared memory so that every global access is a 16-byte row segment
// (thread et then owns row et / 8 and 16 consecutive columns, or 8 SiLU·up outputs).
// Row sums of squares per 32 columns pair two threads' halves; argmax likewise,
// ties to the lowest column.
template <int EPI>
__device__ __forceinline__ void wide_epilogue(const TcArgs& a, const float* v, int m0, int nt, int c, int et,
                                              float* stile) {
#pragma unroll
  for (int t = 0; t < TC_BM; ++t) stile[t * WG_EPI_LD + c] = v[t];
  epi_sync();
  const int t = et >> 3, part = et & 7;
  const int m = m0 + t;
  const bool row_ok = m < a.M;
  const float* src = stile + t * WG_EPI_LD;
  if constexpr (EPI == DFL_EPI_SILU_MUL) {
    // packed per 64 columns as [32 gate | 32 up]: outputs nt*64 + [8*part, 8*part + 8)
    const int oc = part * 8, g = oc >> 5, j = oc & 31;
    const int on = nt * 64 + oc;
    if (row_ok && nt * TC_NT + g * 64 + j < a.N) {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float r2[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float gt = round_bf16(src[g * 64 + j + e + u]);
          const float up = round_bf16(src[g * 64 + 32 + j + e + u]);
          r2[u] = round_bf16(gt / (1.f + __expf(-gt))) * up;
        }
        pk[e / 2] = pack_bf16x2(r2[0], r2[1]);
      }
      *reinterpret_cast<uint4*>(a.y + (long long)m * a.ldy + on) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  } else if constexpr (EPI == DFL_EPI_ARGMAX) {
    const int n0 = nt * TC_NT + part * 16;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float val = n0 + e < a.N ? round_bf16(src[part * 16 + e]) : -INFINITY;
      if (val > best) {  // strictly greater: the lowest column wins ties
        best = val;
        bidx = n0 + e < a.N ? n0 + e : bidx;
      }
    }
    const float ob = __shfl_xor_sync(0xffffffffu, best, 1);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, 1);
    if (ob > best || (ob == best && oi < bidx)) {
      best = ob;
      bidx = oi;
    }
    const int grp = nt * 4 + (part >> 1);
    if (row_ok && !(part & 1) && grp < a.n_groups)
      a.argmax[(long long)m * a.n_groups + grp] = make_float2(best, __int_as_float(bidx));
  } else if constexpr (EPI == DFL_EPI_STORE_F32) {
    const int n0 = nt * TC_NT + part * 16;
    if (row_ok && n0 < a.N) {
      float4* yp = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + (long long)m * a.ldy + n0);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        yp[e] = make_float4(src[part * 16 + 4 * e], src[part * 16 + 4 * e + 1], src[part * 16 + 4 * e + 2],
                            src[part * 16 + 4 * e + 3]);
    }
  } else {
    const int n0 = nt * TC_NT + part * 16;
    const bool ok = row_ok && n0 < a.N;
    float y[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) y[e] = src[part * 16 + e];
    if constexpr (EPI == DFL_EPI_RESIDUAL) {
      uint4 r0 = make_uint4(0, 0, 0, 0), r1 = r0;
      if (ok) {
        const uint4* rp = reinterpret_cast<const uint4*>(a.res + (long long)m * a.ldr + n0);
        r0 = rp[0];
        r1 = rp[1];
      }
      const __nv_bfloat16* rb0 = reinterpret_cast<const __nv_bfloat16*>(&r0);
      const __nv_bfloat16* rb1 = reinterpret_cast<const __nv_bfloat16*>(&r1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        y[e] = bf2f(rb0[e]) + round_bf16(y[e]);
        y[8 + e] = bf2f(rb1[e]) + round_bf16(y[8 + e]);
      }
    }
    uint32_t pk[8];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      pk[e / 2] = pack_bf16x2(y[e], y[e + 1]);
      const float q0 = round_bf16(y[e]), q1 = round_bf16(y[e + 1]);
      ss += q0 * q0 + q1 * q1;
    }
    if (ok) {
      uint4* yp = reinterpret_cast<uint4*>(a.y + (long long)m * a.ldy + n0);
      yp[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      yp[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      if (a.y2) {
        uint4* y2p = reinterpret_cast<uint4*>(a.y2 + (long long)m * a.ldy2 + n0);
        y2p[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        y2p[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
    }
    if (a.sumsq_out) {
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const int grp = nt * 4 + (part >> 1);
      if (row_ok && !(part & 1) && grp < a.n_groups) a.sumsq_out[(long long)m * a.n_groups + grp] = ss;
    }
  }
  epi_sync();  // the transpose tile is rewritten by the next 16 rows
}

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) gemm_wide_kernel(const __grid_constant__ CUtensorMap xmap, WgArgs w) {
  const TcArgs& a = w.t;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int ST = w.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + WG_OFF_BAR);
  uint64_t* empty = full + WG_MAX_STAGES;
  uint64_t* accf = empty + WG_MAX_STAGES;  // [2]
  uint64_t* acce = accf + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + WG_OFF_TMEM);
  float* stile = reinterpret_cast<float*>(smem + WG_OFF_EPI);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bn = w.bn;
  const uint32_t x_bytes = (uint32_t)bn * TC_BK * 2;
  unsigned char* xring = smem + ST * TC_W_BYTES;  // X stage s at xring + s * x_bytes (1024-aligned)
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(TC_NT >> 4) << 24);
  // this CTA's work items (tile x K range): blockIdx.x, blockIdx.x + gridDim.x, ...
  const int items = w.tiles * w.split;
  const int my_tiles = items > (int)blockIdx.x ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const long long my_units = (long long)my_tiles * a.kb;  // upper bound (0 means no work)

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "n"(2 * WG_BN_MAX));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_launch_dependents();

  if (warp == 0) {
    // ---------------- producer: weight units (bulk) + X tiles (TMA) ----------------
    // stage / phase advance incrementally: no integer division on the issue path
    if (lane == 0 && my_units > 0) {
      const uint64_t pol_w = l2_policy_evict_normal();
      const uint64_t pol_x = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      long long i = 0;
      bool ok = true;
      bool waited_dep = false;
      for (int tt = 0; tt < my_tiles && ok; ++tt) {
        const int item = (int)blockIdx.x + tt * (int)gridDim.x;
        const int tl = item / w.split, sp = item % w.split;
        const int nt = tl / w.m_tiles, mt = tl % w.m_tiles;
        const unsigned char* wsrc = a.wt + (long long)nt * a.kb * TC_W_BYTES;
        const int j0 = sp * a.kb / w.split, j1 = (sp + 1) * a.kb / w.split;
        for (int j = j0; j < j1; ++j, ++i) {
          if (i >= ST && !mbar_wait(&empty[s], ph ^ 1u, 221, a.err)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], TC_W_BYTES + x_bytes);
          bulk_load(smem + s * TC_W_BYTES, wsrc + (long long)j * TC_W_BYTES, TC_W_BYTES, &full[s], pol_w);
          if (!waited_dep) {  // X is produced by the previous kernel; weights are not
            grid_dependency_wait();
            waited_dep = true;
          }
          tma_load_2d(&xmap, &full[s], xring + s * x_bytes, j * TC_BK, mt * bn, pol_x);
          if (++s == ST) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // gave up: let the copies already in flight land before the CTA exits
        const long long first = i > ST ? i - ST : 0;
        for (long long k = first; k < i; ++k)
          mbar_wait(&full[k % ST], (uint32_t)((k / ST) & 1), 229, a.err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer: whole K loop of each tile into one accumulator ----------------
    if (lane == 0 && my_units > 0) {
      const uint32_t w0 = smem_u32(smem), x0 = smem_u32(xring);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int tt = 0; tt < my_tiles && ok; ++tt) {
        const int buf = tt & 1;
        const int sp = ((int)blockIdx.x + tt * (int)gridDim.x) % w.split;
        const int j0 = sp * a.kb / w.split, j1 = (sp + 1) * a.kb / w.split;
        if (!mbar_wait(&acce[buf], (uint32_t)((tt >> 1) & 1) ^ 1u, 222, a.err)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * WG_BN_MAX);
        for (int j = j0; j < j1; ++j) {
          if (!mbar_wait(&full[s], ph, 223, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(w0 + s * TC_W_BYTES);
          const uint64_t bd = sw128_desc(x0 + s * x_bytes);
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk)
            tc_mma(d, ad + 2 * kk, bd + 2 * kk, idesc, (j == j0 && kk == 0) ? 0u : 1u);
          tc_commit(&empty[s]);
          if (++s == ST) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(&accf[buf]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;
    grid_dependency_wait();
    TcArgs pa = a;  // split > 1: this item's raw fp32 partial
    pa.ldy = a.N;
    pa.y2 = nullptr;
    pa.sumsq_out = nullptr;
    for (int tt = 0; tt < my_tiles; ++tt) {
      const int item = (int)blockIdx.x + tt * (int)gridDim.x;
      const int tl = item / w.split, sp = item % w.split;
      const int nt = tl / w.m_tiles, mt = tl % w.m_tiles;
      pa.y = reinterpret_cast<__nv_bfloat16*>(w.part + (long long)sp * a.M * a.N);
      const int buf = tt & 1;
      if (!mbar_wait(&accf[buf], (uint32_t)((tt >> 1) & 1), 225, a.err)) break;
      tc_fence_after();
      for (int ch = 0; ch < bn / TC_BM; ++ch) {
        const int m0 = mt * bn + ch * TC_BM;
        if (m0 >= a.M) break;  // uniform over the four warps
        float v[TC_BM];
        tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * WG_BN_MAX + ch * TC_BM), v);
        if (w.split > 1)
          wide_epilogue<DFL_EPI_STORE_F32>(pa, v, m0, nt, q * 32 + lane, threadIdx.x - 32 * TC_EPI_WARP0, stile);
        else
          wide_epilogue<EPI>(a, v, m0, nt, q * 32 + lane, threadIdx.x - 32 * TC_EPI_WARP0, stile);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "n"(2 * WG_BN_MAX));
  }
}

// Split-K completion of the wide GEMM: v = sum over the K ranges in order (fp32), then the
// requested epilogue. One 128-thread block per (128-column tile, 16 rows); thread c owns
// column c, as the tensor-memory layout gives it in the GEMM.
template <int EPI>
__global__ void __launch_bounds__(128) wide_split_reduce_kernel(TcArgs a, const float* __restrict__ part, int split) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  __shared__ float stile[TC_BM * WG_EPI_LD];
  const int nt = blockIdx.x, m0 = blockIdx.y * TC_BM, c = threadIdx.x;
  const int n = nt * TC_NT + c;
  float v[TC_BM];
#pragma unroll
  for (int t = 0; t < TC_BM; ++t) v[t] = 0.f;
  if (n < a.N) {
    for (int sp = 0; sp < split; ++sp) {
      const float* src = part + (long long)sp * a.M * a.N + n;
#pragma unroll
      for (int t = 0; t < TC_BM; ++t)
        if (m0 + t < a.M) v[t] += __ldcg(src + (long long)(m0 + t) * a.N);
    }
  }
  wide_epilogue<EPI>(a, v, m0, nt, c, c, stile);
}

// xn[m, k] = bf16(w[k] * x[m, k] * rsqrt(sum(parts[m]) / K + eps)): the RMSNorm prologue
// of the wide GEMM (partials summed in order, as the fused form does). Grid (M, K / 2048):
// every block recomputes its row's scale and rescales 2048 columns, 8 per thread.
__global__ void __launch_bounds__(256) norm_apply_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                         const __nv_bfloat16* __restrict__ w,
                                                         const float* __restrict__ parts, int n_parts, float eps,
                                                         __nv_bfloat16* __restrict__ xn, int M, int K) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int m = blockIdx.x;
  if (m >= M) return;
  float ss = 0.f;
  for (int p = 0; p < n_parts; ++p) ss += parts[(long long)m * n_parts + p];
  const float inv = rsqrtf(ss / (float)K + eps);
  const int k = blockIdx.y * 2048 + threadIdx.x * 8;
  if (k >= K) return;
  uint4 xv = *reinterpret_cast<const uint4*>(x + (long long)m * ldx + k);
  const uint4 wv = *reinterpret_cast<const uint4*>(w + k);
  __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
  const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
  for (int e = 0; e < 8; ++e) xe[e] = f2bf(bf2f(we[e]) * (bf2f(xe[e]) * inv));
  *reinterpret_cast<uint4*>(xn + (long long)m * K + k) = xv;
}

// ---------------------------------------------------------------------------
// GEMM chain: several M <= 16 weight-streaming GEMMs, each reading the previous one's
// output, in one persistent launch (the projections between two attention calls of a
// verify or draft forward: o_proj -> gate/up -> down -> next layer's qkv).
//
// Each op runs as the stream-K form above (fixed unit ranges per CTA, fp32 partials of
// split tiles summed in range order by the last arriver), so the per-op arithmetic is
// fixed by N, K and the grid. Between ops the launch boundary is replaced by a
// completion counter per op: a CTA adds 1 after its last epilogue store of the op, and
// the X operand of op k + 1 is loaded only once every CTA has done so. Weights do not
// depend on activations: each CTA's producer streams the first ring stages of op k + 1
// before it waits, so the wait and the previous op's epilogue tail overlap the stream.
// When the last op's counter reaches the grid size no CTA waits any more, so the CTA
// that brings it there zeroes every counter for the next launch (which reads them only
// after its grid-dependency wait, i.e. after this launch completed). Loads of data this
// launch wrote (residual rows, RMSNorm partial sums) bypass L1 (ld.global.cg); the X
// tiles come by TMA after a proxy fence on both sides of the counter. Every wait is
// bounded (device error 310 / 311).
// ---------------------------------------------------------------------------
constexpr int CH_MAX_OPS = 6;
constexpr int CH_SITE_DONE = 310;

struct ChainMaps {
  CUtensorMap m[CH_MAX_OPS];
};
struct ChainArgs {
  TcArgs op[CH_MAX_OPS];
  int epi[CH_MAX_OPS];
  int n_ops;
  int* done;   // [CH_MAX_OPS] completion counters (zero between launches)
  int* err;
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;\n" ::: "memory");
}
// bounded wait until every CTA has finished op k of this launch
__device__ __forceinline__ bool chain_wait_done(const ChainArgs& c, int k, int target) {
  if (ld_acquire_gpu(c.done + k) >= target) return true;
  const long long t0 = clock64();
  while (ld_acquire_gpu(c.done + k) < target) {
    if (clock64() - t0 > WAIT_LIMIT_CYCLES) {
      atomicCAS(c.err, 0, CH_SITE_DONE);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void chain_epilogue(int epi, const TcArgs& a, float* v, int nt, int q, int lane, float* xchg) {
  switch (epi) {
    case DFL_EPI_STORE: tc_epilogue<DFL_EPI_STORE>(a, v, 0, nt, q, lane, xchg); break;
    case DFL_EPI_RESIDUAL: tc_epilogue<DFL_EPI_RESIDUAL>(a, v, 0, nt, q, lane, xchg); break;
    case DFL_EPI_SILU_MUL: tc_epilogue<DFL_EPI_SILU_MUL>(a, v, 0, nt, q, lane, xchg); break;
    case DFL_EPI_ARGMAX: tc_epilogue<DFL_EPI_ARGMAX>(a, v, 0, nt, q, lane, xchg); break;
    default: tc_epilogue<DFL_EPI_STORE_F32>(a, v, 0, nt, q, lane, xchg); break;
  }
}

__global__ void __launch_bounds__(TC_THREADS, DFL_TC_MINB)
    gemm_chain_kernel(const __grid_constant__ ChainMaps maps, const __grid_constant__ ChainArgs c) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_OFF_BAR);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* xready = empty + TC_STAGES;
  uint64_t* accf = xready + TC_STAGES;  // [2]
  uint64_t* acce = accf + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TC_OFF_TMEM);
  float* xchg = reinterpret_cast<float*>(smem + TC_OFF_XCHG);
  __nv_bfloat16* s_nw = reinterpret_cast<__nv_bfloat16*>(smem + TC_OFF_NORM);
  __shared__ float s_inv[TC_BM];
  __shared__ int s_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&xready[s], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "n"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_launch_dependents();

  if (warp == 0) {
    // ---------------- producer: weights ahead, X once the previous op is complete ----------------
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      int g = 0;  // ring position over every op's units
      const int target = G;
      bool ok = true;
      for (int k = 0; k < c.n_ops && ok; ++k) {
        const TcArgs& a = c.op[k];
        // an op with fewer units than CTAs runs on its first U1 CTAs (every range non-empty, so
        // the CTAs owning a split tile are consecutive)
        const int Gk = a.U1 < G ? (int)a.U1 : G;
        const long long u0 = cta < Gk ? (long long)cta * a.U1 / Gk : 0;
        const long long u1 = cta < Gk ? (long long)(cta + 1) * a.U1 / Gk : 0;
        const int n_units = (int)(u1 - u0);
        const int pre = n_units < TC_STAGES ? n_units : TC_STAGES;
        for (int i = 0; i < pre && ok; ++i) {
          const int s = (g + i) % TC_STAGES;
          if (g + i >= TC_STAGES && !mbar_wait(&empty[s], (((g + i) / TC_STAGES) & 1) ^ 1, 211, c.err)) ok = false;
          if (!ok) break;
          mbar_expect_tx(&full[s], TC_W_BYTES + TC_X_BYTES);
          bulk_load(smem + s * TC_W_BYTES, a.wt + (u0 + i) * TC_W_BYTES, TC_W_BYTES, &full[s], pol_w);
        }
        if (!ok) break;
        if (k == 0) {
          grid_dependency_wait();  // op 0's X comes from earlier launches
        } else {
          chain_wait_done(c, k - 1, target);
          fence_proxy_async_global();  // generic-proxy stores of op k - 1 -> this CTA's TMA reads
        }
        for (int i = 0; i < pre; ++i)
          tma_load_2d(&maps.m[k], &full[(g + i) % TC_STAGES], smem + TC_OFF_X + ((g + i) % TC_STAGES) * TC_X_BYTES,
                      (int)((u0 + i) % a.kb) * TC_BK, 0, pol_x);
        for (int i = pre; i < n_units; ++i) {
          const int s = (g + i) % TC_STAGES;
          if (!mbar_wait(&empty[s], (((g + i) / TC_STAGES) & 1) ^ 1, 212, c.err)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], TC_W_BYTES + TC_X_BYTES);
          bulk_load(smem + s * TC_W_BYTES, a.wt + (u0 + i) * TC_W_BYTES, TC_W_BYTES, &full[s], pol_w);
          tma_load_2d(&maps.m[k], &full[s], smem + TC_OFF_X + s * TC_X_BYTES, (int)((u0 + i) % a.kb) * TC_BK, 0,
                      pol_x);
        }
        g += n_units;
      }
      if (!ok) {  // gave up: let the copies in flight land before the CTA exits
        for (int i = g > TC_STAGES ? g - TC_STAGES : 0; i < g; ++i)
          mbar_wait(&full[i % TC_STAGES], (i / TC_STAGES) & 1, 219, c.err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t w0 = smem_u32(smem), x0 = smem_u32(smem + TC_OFF_X);
      int g = 0, seg = -1;
      // xready[s] completes only for units of ops with the RMSNorm prologue (the epilogue
      // warps rescale those): its phase is counted per stage over such units
      int xr_uses[TC_STAGES];
#pragma unroll
      for (int s = 0; s < TC_STAGES; ++s) xr_uses[s] = 0;
      bool ok = true;
      for (int k = 0; k < c.n_ops && ok; ++k) {
        const TcArgs& a = c.op[k];
        const bool norm = a.norm_w != nullptr;
        // an op with fewer units than CTAs runs on its first U1 CTAs (every range non-empty, so
        // the CTAs owning a split tile are consecutive)
        const int Gk = a.U1 < G ? (int)a.U1 : G;
        const long long u0 = cta < Gk ? (long long)cta * a.U1 / Gk : 0;
        const long long u1 = cta < Gk ? (long long)(cta + 1) * a.U1 / Gk : 0;
        const int n_units = (int)(u1 - u0);
        for (int i = 0; i < n_units; ++i, ++g) {
          const long long u = u0 + i;
          const int j = (int)(u % a.kb);
          const int s = g % TC_STAGES;
          const bool first = (i == 0) || (j == 0);
          if (first) {
            ++seg;
            if (!mbar_wait(&acce[seg & 1], ((seg >> 1) & 1) ^ 1, 213, c.err)) { ok = false; break; }
            tc_fence_after();
          }
          if (norm) {
            int xr = 0;
#pragma unroll
            for (int ss = 0; ss < TC_STAGES; ++ss)
              if (ss == s) xr = xr_uses[ss]++;
            if (!mbar_wait(&xready[s], xr & 1, 214, c.err)) { ok = false; break; }
          } else if (!mbar_wait(&full[s], (g / TC_STAGES) & 1, 214, c.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)((seg & 1) * TC_NACC * TC_BM);
          const uint64_t ad = sw128_desc(w0 + s * TC_W_BYTES);
          const uint64_t bd = sw128_desc(x0 + s * TC_X_BYTES);
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk)
            tc_mma(d + (uint32_t)((kk % TC_NACC) * TC_BM), ad + 2 * kk, bd + 2 * kk, TC_IDESC,
                   (first && kk < TC_NACC) ? 0u : 1u);
          tc_commit(&empty[s]);
          if (j == a.kb - 1 || i == n_units - 1) tc_commit(&accf[seg & 1]);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps (and the fused RMSNorm rescale) ----------------
    const int et = threadIdx.x - 32 * TC_EPI_WARP0;  // 0..127
    const int q = warp & 3;
    grid_dependency_wait();
    const int target = G;
    int g = 0, seg = -1;
    bool ok = true;
    for (int k = 0; k < c.n_ops; ++k) {
      const TcArgs& a = c.op[k];
      const bool norm = a.norm_w != nullptr;
      // an op with fewer units than CTAs runs on its first U1 CTAs (every range non-empty, so
        // the CTAs owning a split tile are consecutive)
        const int Gk = a.U1 < G ? (int)a.U1 : G;
        const long long u0 = cta < Gk ? (long long)cta * a.U1 / Gk : 0;
        const long long u1 = cta < Gk ? (long long)(cta + 1) * a.U1 / Gk : 0;
      const int n_units = (int)(u1 - u0);
      if (norm && n_units > 0) {
        if (k > 0 && et == 0) chain_wait_done(c, k - 1, target);  // the RMSNorm sums of op k - 1
        epi_sync();  // also: every epilogue thread is done with the previous op's norm weights
        for (int kk = et * 8; kk < a.K; kk += 128 * 8)
          *reinterpret_cast<uint4*>(s_nw + kk) = *reinterpret_cast<const uint4*>(a.norm_w + kk);
        if (et < TC_BM) {
          float ss = 0.f;
          if (et < a.M)
            for (int p = 0; p < a.n_parts; ++p) ss += __ldcg(a.sumsq_in + (long long)et * a.n_parts + p);
          s_inv[et] = rsqrtf(ss / (float)a.K + a.eps);
        }
        epi_sync();
      }
      if (ok)
        for (int i = 0; i < n_units; ++i, ++g) {
          const long long u = u0 + i;
          const int nt = (int)(u / a.kb), j = (int)(u % a.kb);
          const int s = g % TC_STAGES;
          if (i == 0 || j == 0) ++seg;
          if (norm) {
            if (!mbar_wait(&full[s], (g / TC_STAGES) & 1, 215, c.err)) { ok = false; break; }
            const int row = et >> 3, cc = et & 7;
            __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(smem + TC_OFF_X + s * TC_X_BYTES) + row * 64 +
                               ((cc ^ (row & 7)) << 3);
            uint4 xv = *reinterpret_cast<uint4*>(p);
            const uint4 wv = *reinterpret_cast<const uint4*>(s_nw + j * TC_BK + cc * 8);
            __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
            const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
            const float inv = s_inv[row];
#pragma unroll
            for (int e = 0; e < 8; ++e) xe[e] = f2bf(bf2f(we[e]) * (bf2f(xe[e]) * inv));
            *reinterpret_cast<uint4*>(p) = xv;
            fence_proxy_async_smem();
            mbar_arrive(&xready[s]);
          }
          const bool seg_end = (j == a.kb - 1) || (i == n_units - 1);
          if (!seg_end) continue;
          if (!mbar_wait(&accf[seg & 1], (seg >> 1) & 1, 216, c.err)) { ok = false; break; }
          tc_fence_after();
          float v[TC_BM];
          tc_ld_acc(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((seg & 1) * TC_NACC * TC_BM), v);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[seg & 1]);
          const long long tu0 = (long long)nt * a.kb, tu1 = tu0 + a.kb - 1;
          const int c_first = tc_unit_owner(tu0, a.U1, Gk), c_last = tc_unit_owner(tu1, a.U1, Gk);
          bool do_epi = true;
          const int col = q * 32 + lane;
          if (c_first != c_last) {
            const int slot = (nt == (int)(u0 / a.kb)) ? 0 : 1;
            float4* mine = reinterpret_cast<float4*>(a.partial + ((long long)cta * 2 + slot) * TC_PART_FLOATS + col * TC_BM);
#pragma unroll
            for (int t4 = 0; t4 < TC_BM / 4; ++t4)
              mine[t4] = make_float4(v[4 * t4], v[4 * t4 + 1], v[4 * t4 + 2], v[4 * t4 + 3]);
            asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
            epi_sync();
            if (et == 0) {
              int prev;
              asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;\n" : "=r"(prev) : "l"(a.counters + nt) : "memory");
              s_flag = (prev == c_last - c_first);
            }
            epi_sync();
            do_epi = s_flag != 0;
            if (do_epi) {
              asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
#pragma unroll
              for (int t = 0; t < TC_BM; ++t) v[t] = 0.f;
              for (int cs0 = c_first; cs0 <= c_last; cs0 += TC_PB) {
                float4 pb[TC_PB][TC_BM / 4];
#pragma unroll
                for (int kq = 0; kq < TC_PB; ++kq) {
                  const int cs = cs0 + kq;
                  if (cs <= c_last) {
                    const long long cs_u0 = (long long)cs * a.U1 / Gk;
                    const int sl = (nt == (int)(cs_u0 / a.kb)) ? 0 : 1;
                    const float4* src = reinterpret_cast<const float4*>(
                        a.partial + ((long long)cs * 2 + sl) * TC_PART_FLOATS + col * TC_BM);
#pragma unroll
                    for (int t4 = 0; t4 < TC_BM / 4; ++t4) pb[kq][t4] = __ldcg(src + t4);
                  }
                }
#pragma unroll
                for (int kq = 0; kq < TC_PB; ++kq) {
                  if (cs0 + kq <= c_last) {
#pragma unroll
                    for (int t4 = 0; t4 < TC_BM / 4; ++t4) {
                      v[4 * t4] += pb[kq][t4].x;
                      v[4 * t4 + 1] += pb[kq][t4].y;
                      v[4 * t4 + 2] += pb[kq][t4].z;
                      v[4 * t4 + 3] += pb[kq][t4].w;
                    }
                  }
                }
              }
              if (et == 0) a.counters[nt] = 0;
            }
            epi_sync();
          }
          if (do_epi) chain_epilogue(c.epi[k], a, v, nt, q, lane, xchg);
        }
      // op k finished by this CTA: publish (generic stores visible to the async proxy too)
      fence_proxy_async_global();
      asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
      epi_sync();
      if (et == 0) {
        int prev;
        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;\n" : "=r"(prev) : "l"(c.done + k) : "memory");
        if (k == c.n_ops - 1 && prev == target - 1)  // every CTA finished every op: reset for the next launch
          for (int kk = 0; kk < c.n_ops; ++kk) c.done[kk] = 0;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "n"(TC_TMEM_COLS));
  }
}

struct TcPlan {
  int n_tiles, m_tiles, kb, grid1;
  long long U1;
  int S;  // > 0: cluster split-K with S ranks per tile; 0: persistent kernel
};

static TcPlan tc_plan(int M, int N, int K) {
  TcPlan p;
  p.n_tiles = (N + TC_NT - 1) / TC_NT;
  p.m_tiles = (M + TC_BM - 1) / TC_BM;
  p.kb = K / TC_BK;
  p.U1 = (long long)p.n_tiles * p.kb;
  p.grid1 = (int)(p.U1 < TC_GRID ? p.U1 : TC_GRID);
  p.S = 0;
#ifndef DFL_TC_CSK_TILES
#define DFL_TC_CSK_TILES TC_GRID
#endif
  if (p.n_tiles < DFL_TC_CSK_TILES) {  // few tiles: one cluster of S ranks per tile, about one CTA per SM
    int S = (TC_GRID + p.n_tiles / 2) / p.n_tiles;
    if (S > DFL_TC_SMAX) S = DFL_TC_SMAX;
    if (S > p.kb) S = p.kb;
    p.S = S < 1 ? 1 : S;
  }
  return p;
}

}  // namespace dfl

using namespace dfl;

extern "C" size_t dfl_gemm_workspace_bytes(int M, int N, int K, int epilogue) {
  (void)epilogue;
  if (M <= 0 || N <= 0 || K <= 0 || K % TC_BK) return 0;
  TcPlan p = tc_plan(M, N, K);
  return TC_COUNTER_BYTES + (size_t)p.m_tiles * p.grid1 * 2 * TC_PART_FLOATS * sizeof(float);
}

extern "C" int dfl_gemm_argmax_tiles(int N) { return (N + 31) / 32; }

extern "C" size_t dfl_packed_weight_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || K % TC_BK) return 0;
  return (size_t)((N + TC_NT - 1) / TC_NT) * (K / TC_BK) * TC_W_BYTES;
}

extern "C" int dfl_pack_weight_bf16(const void* w, int N, int K, void* out, size_t out_bytes, void* stream) {
  if (!w || !out || N <= 0 || K <= 0 || K % TC_BK || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15)) {
    set_error("dfl_pack_weight_bf16: bad arguments (K %% 64 == 0, 16-byte aligned buffers)");
    return DFL_ERR_INVALID;
  }
  if (out_bytes < dfl_packed_weight_bytes(N, K)) {
    set_error("dfl_pack_weight_bf16: output too small");
    return DFL_ERR_INVALID;
  }
  const long long n_chunks = (long long)dfl_packed_weight_bytes(N, K) / 16;
  const int blocks = (int)((n_chunks + 255) / 256 < 148 * 16 ? (n_chunks + 255) / 256 : 148 * 16);
  pack_weight_kernel<<<blocks, 256, 0, as_stream(stream)>>>(static_cast<const __nv_bfloat16*>(w), N, K,
                                                            static_cast<unsigned char*>(out), n_chunks);
  return check_launch("dfl_pack_weight_bf16");
}

// rope (nullable): fuse the q/k head norm + RoPE + append into the QKV projection when the
// plan is the cluster split-K form over one 16-row tile; *fused reports whether it was
static int gemm_bf16_impl(const void* x, int64_t ldx, const void* w_packed, int M, int N, int K, int epilogue,
                          const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                          void* argmax_partials, const void* norm_w, const float* sumsq_in, int n_parts, float eps,
                          float* sumsq_out, void* workspace, size_t workspace_bytes, void* stream,
                          const QkvArgs* rope = nullptr, bool* fused = nullptr, int rope_layers = 0,
                          const void* const* rope_k_norms = nullptr) {
  if (fused) *fused = false;
  if (M == 0) return DFL_OK;
  const void* w = w_packed;
  if (!x || !w || M < 0 || N <= 0 || K <= 0) {
    set_error("dfl_gemm_bf16: null pointer or bad shape M=%d N=%d K=%d", M, N, K);
    return DFL_ERR_INVALID;
  }
  if (K % TC_BK || N % 32 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15)) {
    set_error("dfl_gemm_bf16: needs K %% 64 == 0, N %% 32 == 0, 16-byte aligned x/w, ldx %% 8 == 0 (K=%d N=%d ldx=%lld)",
              K, N, (long long)ldx);
    return DFL_ERR_UNSUPPORTED;
  }
  if (epilogue == DFL_EPI_ARGMAX) {
    if (!argmax_partials) {
      set_error("dfl_gemm_bf16: argmax epilogue needs argmax_partials");
      return DFL_ERR_INVALID;
    }
  } else if (!y) {
    set_error("dfl_gemm_bf16: y is null");
    return DFL_ERR_INVALID;
  }
  if (epilogue == DFL_EPI_RESIDUAL && !residual) {
    set_error("dfl_gemm_bf16: residual epilogue needs a residual pointer");
    return DFL_ERR_INVALID;
  }
  if (epilogue == DFL_EPI_SILU_MUL && N % 64) {
    set_error("dfl_gemm_bf16: silu-mul epilogue needs N %% 64 == 0 (packed gate/up), N=%d", N);
    return DFL_ERR_UNSUPPORTED;
  }
  if (norm_w && (!sumsq_in || n_parts != K / 32 || K > TC_NORM_MAX_K)) {
    set_error("dfl_gemm_bf16: the fused RMSNorm prologue needs K/32 sumsq_in partials and K <= %d", TC_NORM_MAX_K);
    return DFL_ERR_INVALID;
  }
  TcPlan p = tc_plan(M, N, K);
  if ((size_t)p.m_tiles * p.n_tiles > (size_t)TC_MAX_COUNTERS) {
    set_error("dfl_gemm_bf16: too many output tiles (%d x %d)", p.m_tiles, p.n_tiles);
    return DFL_ERR_UNSUPPORTED;
  }
  const size_t need = dfl_gemm_workspace_bytes(M, N, K, epilogue);
  if (!workspace || workspace_bytes < need) {
    set_error("dfl_gemm_bf16: workspace too small (%zu < %zu bytes)", workspace_bytes, need);
    return DFL_ERR_WORKSPACE;
  }
  const CUtensorMap* xm = tensor_map_2d_bf16(x, M, K, ldx, TC_BM, TC_BK);
  if (!xm) return DFL_ERR_CUDA;

  TcArgs a;
  a.wt = static_cast<const unsigned char*>(w);
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.y2 = static_cast<__nv_bfloat16*>(y2);
  a.ldy2 = ldy2;
  a.argmax = static_cast<float2*>(argmax_partials);
  a.counters = static_cast<int*>(workspace);
  a.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + TC_COUNTER_BYTES);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.sumsq_in = sumsq_in;
  a.n_parts = n_parts;
  a.eps = eps;
  a.sumsq_out = sumsq_out;
  a.err = device_error_word();
  a.n_groups = N / 32;
  a.M = M;
  a.N = N;
  a.K = K;
  a.n_tiles = p.n_tiles;
  a.kb = p.kb;
  a.U1 = p.U1;
  a.grid1 = p.grid1;
  a.rope_on = rope && p.S && p.m_tiles == 1 && epilogue == DFL_EPI_STORE;
  if (a.rope_on) a.rope = *rope;
  else memset(&a.rope, 0, sizeof(a.rope));
  a.rope_layer_heads = 0;
  memset(a.rope_k_norm, 0, sizeof(a.rope_k_norm));
  if (a.rope_on && rope_layers > 0) {
    a.rope_layer_heads = 2 * rope->Hkv;
    for (int l = 0; l < rope_layers; ++l) a.rope_k_norm[l] = static_cast<const __nv_bfloat16*>(rope_k_norms[l]);
  }
  if (fused) *fused = a.rope_on;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = p.S ? dim3(p.S, p.n_tiles, p.m_tiles) : dim3(p.grid1 * p.m_tiles);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TC_SMEM_BASE + (norm_w ? (size_t)K * 2 : 0);
  int recv_off = 0;
  if (p.S) {
    const bool silu = epilogue == DFL_EPI_SILU_MUL;
    const int units = silu ? 2 : 4;
    const int owned = (units + p.S - 1) / p.S;
    const int slots = silu ? 2 * p.S : p.S - 1;
    const size_t recv = (size_t)owned * slots * TC_CSK_SLOT_BYTES;
    const size_t normb = norm_w ? (size_t)K * 2 : 0;
    const size_t ded = CSK_OFF_NORM + normb + recv + 1024;
    if (recv > 0 && 3 * (ded + CSK_RESERVED_PER_CTA) <= (size_t)CSK_SMEM_PER_SM) {
      recv_off = (int)(CSK_OFF_NORM + normb);
      cfg.dynamicSmemBytes = ded;
    } else {
      cfg.dynamicSmemBytes = CSK_OFF_NORM + normb + 1024;
    }
  }
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
#ifdef DFL_NO_PDL
  attr[0].val.programmaticStreamSerializationAllowed = 0;
#else
  attr[0].val.programmaticStreamSerializationAllowed = 1;
#endif
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.S ? p.S : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.S ? 2 : 1;
  cudaError_t err;
  switch (epilogue) {
#define DFL_LAUNCH(E)                                                                                       \
  case E: {                                                                                                 \
    static bool init = false;                                                                               \
    if (!init) {                                                                                            \
      cudaFuncSetAttribute(gemm_tc_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,                  \
                           TC_SMEM_BASE + TC_NORM_MAX_K * 2);                                               \
      cudaFuncSetAttribute(gemm_csk_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,                 \
                           TC_SMEM_BASE + TC_NORM_MAX_K * 2);                                               \
      if (DFL_TC_SMAX > 8) cudaFuncSetAttribute(gemm_csk_kernel<E>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1); \
      init = true;                                                                                          \
    }                                                                                                       \
    err = p.S ? cudaLaunchKernelEx(&cfg, gemm_csk_kernel<E>, *xm, a, p.S, recv_off)                                   \
              : cudaLaunchKernelEx(&cfg, gemm_tc_kernel<E>, *xm, a);                                        \
    break;                                                                                                  \
  }
    DFL_LAUNCH(DFL_EPI_STORE)
    DFL_LAUNCH(DFL_EPI_RESIDUAL)
    DFL_LAUNCH(DFL_EPI_SILU_MUL)
    DFL_LAUNCH(DFL_EPI_ARGMAX)
    DFL_LAUNCH(DFL_EPI_STORE_F32)
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

extern "C" int dfl_gemm_bf16(const void* x, int64_t ldx, const void* w_packed, int M, int N, int K, int epilogue,
                             const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                             void* argmax_partials, const void* norm_w, const float* sumsq_in, int n_parts,
                             float eps, float* sumsq_out, void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_bf16_impl(x, ldx, w_packed, M, N, K, epilogue, residual, ldr, y, ldy, y2, ldy2, argmax_partials, norm_w,
                        sumsq_in, n_parts, eps, sumsq_out, workspace, workspace_bytes, stream);
}

extern "C" int dfl_gemm_qkv_rope(const void* x, int64_t ldx, const void* w_packed, int M, int K, const void* norm_w,
                                 const float* sumsq_in, int n_parts, float eps, void* qkv, int64_t ldqkv,
                                 const int32_t* pos, const int32_t* row_seq, const void* q_norm, const void* k_norm,
                                 const float* inv_freq, void* q_out, void* k_cache, void* v_cache, int64_t seq_stride,
                                 int64_t head_stride, const int32_t* page_table, int64_t pt_stride, int page_size,
                                 int Hq, int Hkv, int hd, void* workspace, size_t workspace_bytes, void* stream) {
  if (M == 0) return DFL_OK;
  if (!pos || !q_norm || !k_norm || !inv_freq || !q_out || !k_cache || !v_cache || Hq <= 0 || Hkv <= 0 || hd <= 0) {
    set_error("dfl_gemm_qkv_rope: null pointer or bad head geometry");
    return DFL_ERR_INVALID;
  }
  QkvArgs r;
  memset(&r, 0, sizeof(r));
  r.qkv = static_cast<const __nv_bfloat16*>(qkv);
  r.ldqkv = ldqkv;
  r.q_stride = hd;
  r.pos = pos;
  r.row_seq = row_seq;
  r.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  r.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  r.inv_freq = inv_freq;
  r.q_out = static_cast<__nv_bfloat16*>(q_out);
  r.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  r.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  r.seq_stride = seq_stride;
  r.head_stride = head_stride;
  r.M = M;
  r.Hq = Hq;
  r.Hkv = Hkv;
  r.hd = hd;
  r.rot_dim = hd;
  r.eps = eps;
  r.do_q = 1;
  r.page_table = page_table;
  r.pt_stride = pt_stride;
  r.page_shift = 0;
  if (page_table) {
    if (page_size < 64 || (page_size & (page_size - 1)) || pt_stride <= 0) {
      set_error("dfl_gemm_qkv_rope: page_size must be a power of two >= 64 (got %d)", page_size);
      return DFL_ERR_INVALID;
    }
    while ((1 << r.page_shift) < page_size) ++r.page_shift;
  }
  const int N = (Hq + 2 * Hkv) * hd;
  bool fused = false;
  const int st = gemm_bf16_impl(x, ldx, w_packed, M, N, K, DFL_EPI_STORE, nullptr, 0, qkv, ldqkv, nullptr, 0, nullptr,
                                norm_w, sumsq_in, n_parts, eps, nullptr, workspace, workspace_bytes, stream,
                                hd == TC_NT ? &r : nullptr, &fused);
  if (st != DFL_OK || fused) return st;
  // another GEMM form: the separate append kernel (the same arithmetic)
  if (page_table)
    return dfl_qkv_rope_append_paged(qkv, ldqkv, hd, pos, row_seq, q_norm, k_norm, inv_freq, q_out, k_cache, v_cache,
                                     seq_stride, head_stride, page_table, pt_stride, page_size, M, Hq, Hkv, hd, hd, eps,
                                     1, stream);
  return dfl_qkv_rope_append(qkv, ldqkv, hd, pos, row_seq, q_norm, k_norm, inv_freq, q_out, k_cache, v_cache,
                             seq_stride, head_stride, M, Hq, Hkv, hd, hd, eps, 1, stream);
}

extern "C" int dfl_gemm_kv_append_layers(const void* x, int64_t ldx, const void* w_packed, int M, int K,
                                         const void* norm_w, const float* sumsq_in, int n_parts, float eps, void* kv,
                                         int64_t ldkv, const int32_t* pos, const int32_t* row_seq,
                                         const void* const* k_norms, const float* inv_freq, void* k_cache,
                                         void* v_cache, int64_t layer_stride, int64_t seq_stride,
                                         int64_t head_stride, const int32_t* page_table, int64_t pt_stride,
                                         int page_size, int n_layers, int Hkv, int hd, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  if (M == 0) return DFL_OK;
  if (!pos || !k_norms || !inv_freq || !k_cache || !v_cache || n_layers <= 0 || n_layers > TC_KV_LAYERS_MAX ||
      Hkv <= 0 || hd <= 0) {
    set_error("dfl_gemm_kv_append_layers: null pointer, bad head geometry or more than %d layers", TC_KV_LAYERS_MAX);
    return DFL_ERR_INVALID;
  }
  for (int l = 0; l < n_layers; ++l)
    if (!k_norms[l]) {
      set_error("dfl_gemm_kv_append_layers: null k_norm of layer %d", l);
      return DFL_ERR_INVALID;
    }
  QkvArgs r;
  memset(&r, 0, sizeof(r));
  r.qkv = static_cast<const __nv_bfloat16*>(kv);
  r.ldqkv = ldkv;
  r.q_stride = hd;
  r.pos = pos;
  r.row_seq = row_seq;
  r.k_norm = static_cast<const __nv_bfloat16*>(k_norms[0]);
  r.q_norm = r.k_norm;
  r.inv_freq = inv_freq;
  r.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  r.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  r.seq_stride = seq_stride;
  r.head_stride = head_stride;
  r.M = M;
  r.Hq = 0;
  r.Hkv = Hkv;
  r.hd = hd;
  r.rot_dim = hd;
  r.eps = eps;
  r.do_q = 0;
  r.page_table = page_table;
  r.pt_stride = pt_stride;
  r.page_shift = 0;
  r.layer_stride = layer_stride;
  if (page_table) {
    if (page_size < 64 || (page_size & (page_size - 1)) || pt_stride <= 0) {
      set_error("dfl_gemm_kv_append_layers: page_size must be a power of two >= 64 (got %d)", page_size);
      return DFL_ERR_INVALID;
    }
    while ((1 << r.page_shift) < page_size) ++r.page_shift;
  }
  const int per = 2 * Hkv * hd;
  bool fused = false;
  const int st = gemm_bf16_impl(x, ldx, w_packed, M, n_layers * per, K, DFL_EPI_STORE, nullptr, 0, kv, ldkv, nullptr, 0,
                                nullptr, norm_w, sumsq_in, n_parts, eps, nullptr, workspace, workspace_bytes, stream,
                                hd == TC_NT ? &r : nullptr, &fused, n_layers, k_norms);
  if (st != DFL_OK || fused) return st;
  // another GEMM form: one append launch per layer (the same arithmetic)
  char* kb = static_cast<char*>(k_cache);
  char* vb = static_cast<char*>(v_cache);
  for (int l = 0; l < n_layers; ++l) {
    const void* kvl = static_cast<const char*>(kv) + (size_t)l * per * 2;
    void* kl = kb + (size_t)l * layer_stride * 2;
    void* vl = vb + (size_t)l * layer_stride * 2;
    const int s = page_table
                      ? dfl_qkv_rope_append_paged(kvl, ldkv, hd, pos, row_seq, k_norms[l], k_norms[l], inv_freq,
                                                  nullptr, kl, vl, seq_stride, head_stride, page_table, pt_stride,
                                                  page_size, M, 0, Hkv, hd, hd, eps, 0, stream)
                      : dfl_qkv_rope_append(kvl, ldkv, hd, pos, row_seq, k_norms[l], k_norms[l], inv_freq, nullptr,
                                            kl, vl, seq_stride, head_stride, M, 0, Hkv, hd, hd, eps, 0, stream);
    if (s != DFL_OK) return s;
  }
  return DFL_OK;
}

extern "C" int dfl_gemm_qkv_rope_launches(int M, int K, int Hq, int Hkv, int hd) {
  if (M <= 0 || K <= 0 || K % TC_BK || Hq < 0 || Hkv <= 0 || hd <= 0) return -1;
  const TcPlan p = tc_plan(M, (Hq + 2 * Hkv) * hd, K);
  return (hd == TC_NT && p.S && p.m_tiles == 1) ? 1 : 2;
}

static int wide_split_of(int K, int k_split) {
  const int kb = K / TC_BK;
  return k_split < 1 ? 1 : (k_split > kb ? kb : k_split);
}

extern "C" size_t dfl_gemm_wide_workspace_bytes(int M, int N, int K, int with_norm, int k_split) {
  if (M <= 0 || N <= 0 || K <= 0 || K % TC_BK) return 0;
  const size_t xn = with_norm ? (((size_t)M * K * 2 + 255) & ~(size_t)255) : 0;
  const int S = wide_split_of(K, k_split);
  return xn + (S > 1 ? (size_t)S * M * N * 4 : 0);
}

extern "C" int dfl_gemm_bf16_wide(const void* x, int64_t ldx, const void* w_packed, int M, int N, int K, int epilogue,
                                  const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2, int64_t ldy2,
                                  void* argmax_partials, const void* norm_w, const float* sumsq_in, int n_parts,
                                  float eps, float* sumsq_out, int k_split, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  if (M == 0) return DFL_OK;
  const void* w = w_packed;
  if (!x || !w || M < 0 || N <= 0 || K <= 0) {
    set_error("dfl_gemm_bf16_wide: null pointer or bad shape M=%d N=%d K=%d", M, N, K);
    return DFL_ERR_INVALID;
  }
  if (K % TC_BK || N % 32 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15)) {
    set_error("dfl_gemm_bf16_wide: needs K %% 64 == 0, N %% 32 == 0, 16-byte aligned x/w, ldx %% 8 == 0");
    return DFL_ERR_UNSUPPORTED;
  }
  if (epilogue == DFL_EPI_ARGMAX ? !argmax_partials : !y) {
    set_error("dfl_gemm_bf16_wide: missing output pointer");
    return DFL_ERR_INVALID;
  }
  const bool raw_partials = epilogue == DFL_EPI_PARTIALS;
  if (raw_partials) {
    if (ldy != N) {
      set_error("dfl_gemm_bf16_wide: the partials epilogue writes [k_split][M][N] slabs (ldy must be N)");
      return DFL_ERR_INVALID;
    }
    epilogue = DFL_EPI_STORE_F32;
  }
  if (epilogue == DFL_EPI_RESIDUAL && !residual) {
    set_error("dfl_gemm_bf16_wide: residual epilogue needs a residual pointer");
    return DFL_ERR_INVALID;
  }
  if (epilogue == DFL_EPI_SILU_MUL && N % 64) {
    set_error("dfl_gemm_bf16_wide: silu-mul epilogue needs N %% 64 == 0 (packed gate/up), N=%d", N);
    return DFL_ERR_UNSUPPORTED;
  }
  // the epilogue moves 16-byte row segments of y / y2 / residual
  const uintptr_t mis = reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(y2) |
                        reinterpret_cast<uintptr_t>(residual);
  if ((mis & 15) || ldy % 8 || (y2 && ldy2 % 8) || (residual && ldr % 8)) {
    set_error("dfl_gemm_bf16_wide: y / y2 / residual must be 16-byte aligned with row strides %% 8 == 0");
    return DFL_ERR_UNSUPPORTED;
  }
  if (norm_w && (!sumsq_in || n_parts != K / 32)) {
    set_error("dfl_gemm_bf16_wide: the RMSNorm prologue needs K/32 sumsq_in partials");
    return DFL_ERR_INVALID;
  }
  const int split = wide_split_of(K, k_split);
  const size_t need = dfl_gemm_wide_workspace_bytes(M, N, K, norm_w != nullptr, raw_partials ? 1 : split);
  if (need && (!workspace || workspace_bytes < need)) {
    set_error("dfl_gemm_bf16_wide: workspace too small (%zu < %zu bytes)", workspace_bytes, need);
    return DFL_ERR_WORKSPACE;
  }
  cudaStream_t st = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const void* xs = x;
  long long ldxs = ldx;
  if (norm_w) {
    cudaLaunchConfig_t nc = {};
    nc.gridDim = dim3(M, (K + 2047) / 2048);
    nc.blockDim = dim3(256);
    nc.stream = st;
    nc.attrs = attr;
    nc.numAttrs = 1;
    __nv_bfloat16* xn = static_cast<__nv_bfloat16*>(workspace);
    cudaError_t e = cudaLaunchKernelEx(&nc, norm_apply_kernel, static_cast<const __nv_bfloat16*>(x), (long long)ldx,
                                       static_cast<const __nv_bfloat16*>(norm_w), sumsq_in, n_parts, eps, xn, M, K);
    if (e != cudaSuccess) {
      set_error("dfl_gemm_bf16_wide: norm launch failed: %s", cudaGetErrorString(e));
      return DFL_ERR_CUDA;
    }
    xs = xn;
    ldxs = K;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // tokens per tile: all rows up to 256; above that the width among 256 / 192 / 160 / 128
  // with the least modelled time per SM: waves x (448 + width), the constant being the
  // weight-unit share of a k-step measured on B200 (narrow tiles re-read W from L2).
  // 160 puts the 20-tile o_proj weights of a 1024-row batch on 140 of 148 SMs in one wave
  // (256 leaves 68 idle): 33.4 against 34.8 us on B200
  const int n_tiles = (N + TC_NT - 1) / TC_NT;
  int bn = M >= WG_BN_MAX ? WG_BN_MAX : (M + TC_BM - 1) / TC_BM * TC_BM;
  if (M > WG_BN_MAX) {
    long long best = -1;
    for (int cand : {256, 192, 160, 128}) {
      const long long tiles = (long long)n_tiles * ((M + cand - 1) / cand);
      const long long cost = (tiles + sms - 1) / sms * (448 + cand);
      if (best < 0 || cost < best) {
        best = cost;
        bn = cand;
      }
    }
  }
  const CUtensorMap* xm = tensor_map_2d_bf16(xs, M, K, ldxs, bn, TC_BK);
  if (!xm) return DFL_ERR_CUDA;
  WgArgs wa;
  TcArgs& a = wa.t;
  a.wt = static_cast<const unsigned char*>(w);
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.y2 = static_cast<__nv_bfloat16*>(y2);
  a.ldy2 = ldy2;
  a.argmax = static_cast<float2*>(argmax_partials);
  a.partial = nullptr;
  a.counters = nullptr;
  a.norm_w = nullptr;
  a.sumsq_in = nullptr;
  a.n_parts = 0;
  a.eps = eps;
  a.sumsq_out = sumsq_out;
  a.err = device_error_word();
  a.n_groups = N / 32;
  a.M = M;
  a.N = N;
  a.K = K;
  a.n_tiles = (N + TC_NT - 1) / TC_NT;
  a.kb = K / TC_BK;
  a.U1 = 0;
  a.grid1 = 0;
  wa.split = split;
  wa.part = split <= 1 ? nullptr
             : raw_partials ? static_cast<float*>(y)
                            : reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                                       (norm_w ? (((size_t)M * K * 2 + 255) & ~(size_t)255) : 0));
  wa.bn = bn;
  wa.stages = WG_RING_BYTES / (TC_W_BYTES + bn * TC_BK * 2);
  if (wa.stages > WG_MAX_STAGES) wa.stages = WG_MAX_STAGES;
  wa.m_tiles = (M + bn - 1) / bn;
  wa.tiles = a.n_tiles * wa.m_tiles;
  const int items = wa.tiles * split;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(items < sms ? items : sms);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = WG_SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err;
  switch (epilogue) {
#define DFL_LAUNCH_WIDE(E)                                                                                  \
  case E: {                                                                                                 \
    static bool init[64] = {false};                                                                         \
    if (dev >= 0 && dev < 64 && !init[dev]) {                                                               \
      cudaFuncSetAttribute(gemm_wide_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, WG_SMEM);      \
      init[dev] = true;                                                                                     \
    }                                                                                                       \
    err = cudaLaunchKernelEx(&cfg, gemm_wide_kernel<E>, *xm, wa);                                           \
    if (err == cudaSuccess && split > 1 && !raw_partials) {                                                 \
      cudaLaunchConfig_t rc = cfg;                                                                          \
      rc.gridDim = dim3(a.n_tiles, (M + TC_BM - 1) / TC_BM);                                                \
      rc.blockDim = dim3(128);                                                                              \
      rc.dynamicSmemBytes = 0;                                                                              \
      err = cudaLaunchKernelEx(&rc, wide_split_reduce_kernel<E>, a, static_cast<const float*>(wa.part), split); \
    }                                                                                                       \
    break;                                                                                                  \
  }
    DFL_LAUNCH_WIDE(DFL_EPI_STORE)
    DFL_LAUNCH_WIDE(DFL_EPI_RESIDUAL)
    DFL_LAUNCH_WIDE(DFL_EPI_SILU_MUL)
    DFL_LAUNCH_WIDE(DFL_EPI_ARGMAX)
    DFL_LAUNCH_WIDE(DFL_EPI_STORE_F32)
#undef DFL_LAUNCH_WIDE
    default:
      set_error("dfl_gemm_bf16_wide: unknown epilogue %d", epilogue);
      return DFL_ERR_INVALID;
  }
  if (err != cudaSuccess) {
    set_error("dfl_gemm_bf16_wide: launch failed: %s", cudaGetErrorString(err));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_device_error(int* code, int clear, void* stream) {
  if (!code) return DFL_ERR_INVALID;
  int* word = device_error_word();
  if (!word) {
    set_error("dfl_device_error: no device error word");
    return DFL_ERR_CUDA;
  }
  cudaError_t e = cudaMemcpyAsync(code, word, sizeof(int), cudaMemcpyDeviceToHost, as_stream(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(word, 0, sizeof(int), as_stream(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  if (e != cudaSuccess) {
    set_error("dfl_device_error: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of dfl_gemm_bf16.
//
// Some callers cannot allocate device memory at all: code that runs inside a
// host callback or a signal-safe path, plugins whose host application owns every
// allocation, or engines that have sized the whole device up front and forbid
// cudaMalloc after start-up. For them the split-K scratch (arrival counters +
// partial tiles) comes from a fixed array compiled into this library instead of a
// caller-provided workspace. The array is sized for one 16-row tile of X (the
// decode shape: M <= 16); larger M is rejected. Every GPU that loads the library
// holds it (about 5.4 MB) until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t NA_SCRATCH_BYTES = TC_COUNTER_BYTES + (size_t)TC_GRID * 2 * TC_PART_FLOATS * sizeof(float);
static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_SCRATCH_BYTES];

// Device address of the scratch array on the current device, looked up once per
// device (the symbol name itself is only a host-side stand-in, never a device pointer).
static void* noalloc_scratch_ptr() {
  static void* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

extern "C" size_t dfl_gemm_noalloc_scratch_bytes(void) { return NA_SCRATCH_BYTES; }

extern "C" int dfl_gemm_bf16_noalloc(const void* x, int64_t ldx, const void* w_packed, int M, int N, int K,
                                     int epilogue, const void* residual, int64_t ldr, void* y, int64_t ldy, void* y2,
                                     int64_t ldy2, void* argmax_partials, const void* norm_w, const float* sumsq_in,
                                     int n_parts, float eps, float* sumsq_out, void* stream) {
  if (M < 0 || N < 0 || K < 0) {
    set_error("dfl_gemm_bf16_noalloc: negative size (M=%d N=%d K=%d)", M, N, K);
    return DFL_ERR_INVALID;
  }
  if (M > TC_BM) {
    set_error("dfl_gemm_bf16_noalloc: M=%d exceeds the built-in scratch limit of %d rows; use dfl_gemm_bf16 with a "
              "workspace",
              M, TC_BM);
    return DFL_ERR_UNSUPPORTED;
  }
  if (M > 0 && N > 0 && K > 0 && K % TC_BK == 0 && dfl_gemm_workspace_bytes(M, N, K, epilogue) > NA_SCRATCH_BYTES) {
    set_error("dfl_gemm_bf16_noalloc: shape M=%d N=%d K=%d needs more scratch than the built-in %zu bytes", M, N, K,
              NA_SCRATCH_BYTES);
    return DFL_ERR_UNSUPPORTED;
  }
  void* scratch = noalloc_scratch_ptr();
  if (!scratch) {
    set_error("dfl_gemm_bf16_noalloc: cudaGetSymbolAddress of the built-in scratch failed");
    return DFL_ERR_CUDA;
  }
  // the arrival counters must start at zero (a call that gave up may have left them set)
  cudaError_t e = cudaMemsetAsync(scratch, 0, TC_COUNTER_BYTES, as_stream(stream));
  if (e != cudaSuccess) {
    set_error("dfl_gemm_bf16_noalloc: clearing the scratch counters failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return dfl_gemm_bf16(x, ldx, w_packed, M, N, K, epilogue, residual, ldr, y, ldy, y2, ldy2, argmax_partials, norm_w,
                       sumsq_in, n_parts, eps, sumsq_out, scratch, NA_SCRATCH_BYTES, stream);
}


// Chain scratch, one fixed layout for every op list (launches with different lists share
// a workspace, and a tile counter must never land on another launch's partial tiles):
// [256 B: per-op completion counters][CH_MAX_TILES ints: tile counters][partial tiles].
constexpr int CH_MAX_TILES = 1 << 16;
constexpr size_t CH_OFF_COUNTERS = 256;
constexpr size_t CH_OFF_PARTIAL = CH_OFF_COUNTERS + (size_t)CH_MAX_TILES * sizeof(int);

extern "C" size_t dfl_gemm_chain_workspace_bytes(const dfl_gemm_op* ops, int n_ops) {
  if (!ops || n_ops <= 0 || n_ops > CH_MAX_OPS) return 0;
  return CH_OFF_PARTIAL + (size_t)TC_GRID * 2 * TC_PART_FLOATS * sizeof(float);
}

extern "C" int dfl_gemm_chain(const dfl_gemm_op* ops, int n_ops, void* workspace, size_t workspace_bytes,
                              void* stream) {
  if (!ops || n_ops <= 0 || n_ops > CH_MAX_OPS) {
    set_error("dfl_gemm_chain: 1..%d ops", CH_MAX_OPS);
    return DFL_ERR_INVALID;
  }
  const size_t need = dfl_gemm_chain_workspace_bytes(ops, n_ops);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    set_error("dfl_gemm_chain: workspace too small or unaligned (%zu < %zu bytes)", workspace_bytes, need);
    return DFL_ERR_WORKSPACE;
  }
  ChainMaps maps;
  ChainArgs c;
  std::memset(&maps, 0, sizeof(maps));
  std::memset(&c, 0, sizeof(c));
  char* ws = static_cast<char*>(workspace);
  c.done = reinterpret_cast<int*>(ws);
  int* counters = reinterpret_cast<int*>(ws + CH_OFF_COUNTERS);
  size_t tiles = 0;
  for (int k = 0; k < n_ops; ++k) tiles += (size_t)(ops[k].N + TC_NT - 1) / TC_NT;
  if (tiles > (size_t)CH_MAX_TILES) {
    set_error("dfl_gemm_chain: %zu output tiles over all ops (at most %d)", tiles, CH_MAX_TILES);
    return DFL_ERR_UNSUPPORTED;
  }
  float* partial = reinterpret_cast<float*>(ws + CH_OFF_PARTIAL);
  c.err = device_error_word();
  c.n_ops = n_ops;
  int max_norm_k = 0;
  for (int k = 0; k < n_ops; ++k) {
    const dfl_gemm_op& o = ops[k];
    const int epi = o.epilogue;
    if (!o.x || !o.w_packed || o.M <= 0 || o.M > TC_BM || o.N <= 0 || o.K <= 0 || o.K % TC_BK || o.N % 32 ||
        o.ldx % 8 || (reinterpret_cast<uintptr_t>(o.x) & 15) || (reinterpret_cast<uintptr_t>(o.w_packed) & 15)) {
      set_error("dfl_gemm_chain: op %d: needs 1 <= M <= %d, K %% 64 == 0, N %% 32 == 0, 16-byte aligned x / w", k,
                TC_BM);
      return DFL_ERR_UNSUPPORTED;
    }
    if (epi < DFL_EPI_STORE || epi > DFL_EPI_STORE_F32 || (epi == DFL_EPI_ARGMAX && !o.argmax_partials) ||
        (epi != DFL_EPI_ARGMAX && !o.y) || (epi == DFL_EPI_RESIDUAL && !o.residual) ||
        (epi == DFL_EPI_SILU_MUL && o.N % 64)) {
      set_error("dfl_gemm_chain: op %d: bad epilogue %d or missing output / residual", k, epi);
      return DFL_ERR_INVALID;
    }
    if (o.norm_w && (!o.sumsq_in || o.n_parts != o.K / 32 || o.K > TC_NORM_MAX_K)) {
      set_error("dfl_gemm_chain: op %d: the RMSNorm prologue needs K/32 sumsq_in partials and K <= %d", k,
                TC_NORM_MAX_K);
      return DFL_ERR_INVALID;
    }
    const CUtensorMap* xm = tensor_map_2d_bf16(o.x, o.M, o.K, o.ldx, TC_BM, TC_BK);
    if (!xm) return DFL_ERR_CUDA;
    maps.m[k] = *xm;
    TcArgs& a = c.op[k];
    a.wt = static_cast<const unsigned char*>(o.w_packed);
    a.res = static_cast<const __nv_bfloat16*>(o.residual);
    a.ldr = o.ldr;
    a.y = static_cast<__nv_bfloat16*>(o.y);
    a.ldy = o.ldy;
    a.y2 = static_cast<__nv_bfloat16*>(o.y2);
    a.ldy2 = o.ldy2;
    a.argmax = static_cast<float2*>(o.argmax_partials);
    a.counters = counters;
    a.partial = partial;
    a.norm_w = static_cast<const __nv_bfloat16*>(o.norm_w);
    a.sumsq_in = o.sumsq_in;
    a.n_parts = o.n_parts;
    a.eps = o.eps;
    a.sumsq_out = o.sumsq_out;
    a.err = c.err;
    a.n_groups = o.N / 32;
    a.M = o.M;
    a.N = o.N;
    a.K = o.K;
    a.n_tiles = (o.N + TC_NT - 1) / TC_NT;
    a.kb = o.K / TC_BK;
    a.U1 = (long long)a.n_tiles * a.kb;
    a.grid1 = TC_GRID;
    c.epi[k] = epi;
    counters += a.n_tiles;
    if (o.norm_w && o.K > max_norm_k) max_norm_k = o.K;
  }
  static bool init[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !init[dev]) {
    cudaFuncSetAttribute(gemm_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         TC_SMEM_BASE + TC_NORM_MAX_K * 2);
    init[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(TC_GRID);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TC_SMEM_BASE + (size_t)max_norm_k * 2;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_chain_kernel, maps, c);
  if (e != cudaSuccess) {
    set_error("dfl_gemm_chain: launch failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}
