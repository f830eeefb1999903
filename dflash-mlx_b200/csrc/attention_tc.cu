// Grouped-query attention on the 5th-generation tensor cores (tcgen05 + TMEM, K/V by TMA),
// head_dim 128: the verify and draft attention of the Qwen3 family
// (mx.fast.scaled_dot_product_attention at adapters.py:620 and draft.py:149-157).
//
// Same work split, masking, key chunks and partial-result format as attn_chunk_kernel
// (attention.cu): one CTA per (key chunk, kv head, 16-row tile segment); its G query heads
// x 16 rows form the rows 0 .. 16G-1 of a 128-row MMA tile (the rest zero). Per 64-key
// block of the chunk:
//   S = Q K^T       tcgen05.mma, M = 128 rows, N = 64 keys, K = 128 dims, into TMEM
//   P = exp2(S - m) softmax warps, one thread per row (TMEM lane), written to one of two
//                   shared-memory buffers (the next block's softmax overlaps this block's
//                   P V) as a bf16 high part and a bf16 low part (about 16 significant
//                   bits: the reference's fp32 softmax weights, not a single bf16 rounding)
//   O += P V        tcgen05.mma, N = 128 dims, K = 64 keys, twice (high, low), in TMEM
// The running maximum is rescaled lazily: O and the row sum are rescaled only when a
// row's maximum grows by more than 8 (log2 units) over the one the exponentials use, and
// the final division and the chunk merge use that maximum -- exact, and the same for a
// row whatever other rows share the tile. V arrives from the cache as [key][dim] and the
// P V product reads it so, as an MN-major B operand (no transpose).
// Warp roles: 0 TMA producer, 1 MMA issuer, 2-3 idle, 4-5 softmax and epilogue.
// K/V come through 3-D tensor maps (dims, key rows, (sequence or page) x kv head planes),
// so a block past a head's last row reads zeros instead of another head's keys. Every
// wait is bounded (device error 320-329).
#include "common.cuh"
#include "tcgen05.cuh"
#include "tma_util.cuh"

#include <cstdlib>
#include <mutex>
#include <unordered_map>

namespace dfl {

constexpr int AT_KB = 64;                 // keys per block
constexpr int AT_HD = 128;                // head dim
constexpr int AT_UNIT = 128 * 128;        // one [128 rows x 128 B] swizzled unit (16 KB)
constexpr int AT_OFF_Q = 0;               // 2 units: dims 0-63, 64-127
constexpr int AT_OFF_K = 2 * AT_UNIT;     // 2 stages x 2 halves x [64 keys x 128 B]
constexpr int AT_OFF_V = 4 * AT_UNIT;     // 2 stages x 2 halves x [64 keys x 128 B]
constexpr int AT_OFF_P = 6 * AT_UNIT;     // 2 buffers x (high unit, low unit)
constexpr int AT_OFF_BAR = 10 * AT_UNIT;
constexpr int AT_NBAR = 24;
constexpr int AT_SMEM = AT_OFF_BAR + AT_NBAR * 8 + 16 + 1024;
constexpr int AT_THREADS = 192;
constexpr uint32_t AT_TMEM_COLS = 256;    // S double buffer (2 x 64) + O (128)
// kind::f16, A = B = bf16, D = f32, K-major; M = 128; N = 64 (S) or 128 (O)
constexpr uint32_t AT_IDESC_S = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t AT_IDESC_O = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(128 >> 3) << 17) |
                                  ((uint32_t)(128 >> 4) << 24);  // B (V) MN-major
constexpr float AT_RESCALE = 8.f;         // lazy rescale threshold (log2 units)

struct AttnTcArgs {
  const __nv_bfloat16* q;  // [M][Hq][128]
  const int* pos;
  const int* row_seq;
  const int* kv_len;
  const int* page_table;   // nullable
  long long pt_stride;
  int page_shift;
  int planes_per_seq;      // contiguous: Hkv (plane = seq * Hkv + h); paged: Hkv (plane = page * Hkv + h)
  float* part_o;
  float2* part_ml;
  __nv_bfloat16* out;
  long long ldo;
  int M, Hq, Hkv, G, causal, n_chunks, segs, key_chunk, direct;
  float scale_log2;
  int* err;
};

struct AttnTcMaps {
  CUtensorMap k, v;
};

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];\n" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// byte offset of element (row r, 16-byte chunk c) in a [rows x 128 B] 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__global__ void __launch_bounds__(AT_THREADS, 1) attn_tc_kernel(const __grid_constant__ AttnTcMaps maps,
                                                                const __grid_constant__ AttnTcArgs a) {
  grid_dependency_launch_dependents();
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AT_OFF_BAR);
  uint64_t* k_full = bars;       // [2]
  uint64_t* k_empty = bars + 2;  // [2]
  uint64_t* v_full = bars + 4;   // [2]
  uint64_t* v_empty = bars + 6;  // [2] MMA commit (the P V products read the stage)
  uint64_t* s_full = bars + 12;  // [2] MMA commit
  uint64_t* s_free = bars + 14;  // [2] 64 softmax arrivals
  uint64_t* p_full = bars + 16;  // [2] 64 softmax arrivals
  uint64_t* p_free = bars + 18;  // [2] MMA commit (also: O complete up to that block)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + AT_OFF_BAR + AT_NBAR * 8);

  __shared__ int s_lim[16];
  __shared__ int s_seq;
  const int chunk = blockIdx.x, kvh = blockIdx.y, tile = blockIdx.z / a.segs, seg = blockIdx.z % a.segs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = tile * 16;

  grid_dependency_wait();  // q, positions and the cache rows come from earlier kernels
  if (threadIdx.x < 32) {  // the tile's rows of this CTA's sequence (as attn_chunk_kernel)
    const int r = threadIdx.x;
    const int m = m0 + r;
    const int p = (r < 16 && m < a.M) ? a.pos[m] : -1;
    const int sq = (r < 16 && m < a.M && a.row_seq) ? a.row_seq[m] : 0;
    bool first = p >= 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int pj = __shfl_sync(0xffffffffu, p, j), sj = __shfl_sync(0xffffffffu, sq, j);
      if (j < r && pj >= 0 && sj == sq) first = false;
    }
    const unsigned firsts = __ballot_sync(0xffffffffu, first);
    const int n = __popc(firsts);
    int row = -1;
    if (seg < n) {
      unsigned msk = firsts;
      for (int k = 0; k < seg; ++k) msk &= msk - 1;
      row = __ffs(msk) - 1;
    }
    const int chosen = __shfl_sync(0xffffffffu, sq, row < 0 ? 0 : row);
    if (r == 0) {
      if (seg == 0 && n > a.segs && chunk == 0 && kvh == 0 && a.err) atomicCAS(a.err, 0, 301);
      s_seq = row < 0 ? -1 : chosen;
    }
    if (r < 16) {
      const bool mine = row >= 0 && p >= 0 && sq == chosen;
      s_lim[r] = !mine ? 0 : (a.causal ? p + 1 : a.kv_len[chosen]);
    }
  }
  __syncthreads();
  if (s_seq < 0) return;
  int lim_max = 0;
#pragma unroll
  for (int r = 0; r < 16; ++r) lim_max = max(lim_max, s_lim[r]);
  const int k_begin = chunk * a.key_chunk;
  if (k_begin >= lim_max) return;
  const int k_end = min(k_begin + a.key_chunk, lim_max);
  const int n_blocks = (k_end - k_begin + AT_KB - 1) / AT_KB;
  const int G = a.G;

  // Q tile (rows hl * 16 + r) and zero padding rows; P padding rows zeroed once
  {
    for (int idx = threadIdx.x; idx < 128 * 16; idx += AT_THREADS) {
      const int row = idx >> 4, c = idx & 15;  // c: 16-byte chunk of the 256-byte row
      uint4 v = make_uint4(0, 0, 0, 0);
      const int hl = row >> 4, r = row & 15;
      if (hl < G && s_lim[r] > 0)
        v = *reinterpret_cast<const uint4*>(a.q + ((long long)(m0 + r) * a.Hq + kvh * G + hl) * AT_HD + c * 8);
      *reinterpret_cast<uint4*>(smem + AT_OFF_Q + (c >> 3) * AT_UNIT + sw_off(row, c & 7)) = v;
    }
    for (int idx = threadIdx.x; idx < 4 * 64 * 8; idx += AT_THREADS) {  // P rows 64-127, all four units
      const int u = idx / 512, rr = 64 + (idx % 512) / 8, c = idx % 8;
      *reinterpret_cast<uint4*>(smem + AT_OFF_P + u * AT_UNIT + sw_off(rr, c)) = make_uint4(0, 0, 0, 0);
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 64);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&p_full[s], 64);
      mbar_init(&p_free[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "n"(AT_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  fence_proxy_async_smem();  // Q / P padding written by generic stores, read by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o = tmem + 128;  // O columns 128-255

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n_blocks; ++i) {
        const int s = i & 1;
        const int key = k_begin + i * AT_KB;
        int plane, row;
        if (a.page_table) {
          plane = a.page_table[s_seq * a.pt_stride + (key >> a.page_shift)] * a.planes_per_seq + kvh;
          row = key & ((1 << a.page_shift) - 1);
        } else {
          plane = s_seq * a.planes_per_seq + kvh;
          row = key;
        }
        if (!mbar_wait(&k_empty[s], ((i >> 1) & 1) ^ 1, 320, a.err)) break;
        mbar_expect_tx(&k_full[s], 2 * 64 * 128);
        for (int h = 0; h < 2; ++h)
          tma_load_3d(&maps.k, &k_full[s], smem + AT_OFF_K + s * 2 * 8192 + h * 8192, h * 64, row, plane);
        if (!mbar_wait(&v_empty[s], ((i >> 1) & 1) ^ 1, 321, a.err)) {
          issued = -(i + 1);
          break;
        }
        mbar_expect_tx(&v_full[s], 2 * 64 * 128);
        for (int h = 0; h < 2; ++h)
          tma_load_3d(&maps.v, &v_full[s], smem + AT_OFF_V + s * 2 * 8192 + h * 8192, h * 64, row, plane);
        issued = i + 1;
      }
      (void)issued;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t q0 = smem_u32(smem + AT_OFF_Q);
      auto mma2 = [&](int j) -> bool {  // O += P V for block j (high, then low part of P)
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, 322, a.err)) return false;
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, 323, a.err)) return false;
        tc_fence_after();
        // V as loaded, [key][dim] in two 64-dim halves of 8 KB: MN-major B, atoms of 8 keys x
        // 64 dims (1 KB) -- the next 8 keys 1 KB on, the next 64 dims 8 KB on; 16 keys a step
        const uint32_t vb = smem_u32(smem + AT_OFF_V + (j & 1) * 2 * 8192);
        for (int part = 0; part < 2; ++part) {
          const uint32_t p0 = smem_u32(smem + AT_OFF_P + ((j & 1) * 2 + part) * AT_UNIT);
#pragma unroll
          for (int kk = 0; kk < AT_KB / 16; ++kk)
            tc_mma(t_o, sw128_desc(p0) + 2 * kk, sw128_mn_desc(vb + kk * 2048, 8192, 1024), AT_IDESC_O,
                   (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&p_free[j & 1]);
        tc_commit(&v_empty[j & 1]);
        return true;
      };
      bool ok = true;
      for (int i = 0; i < n_blocks && ok; ++i) {
        const int s = i & 1;
        if (!mbar_wait(&k_full[s], (i >> 1) & 1, 324, a.err)) break;
        if (!mbar_wait(&s_free[s], ((i >> 1) & 1) ^ 1, 325, a.err)) break;
        tc_fence_after();
        const uint32_t kt = smem_u32(smem + AT_OFF_K + s * 2 * 8192);
        const uint32_t ts = tmem + (uint32_t)(s * 64);
#pragma unroll
        for (int kk = 0; kk < AT_HD / 16; ++kk)  // 8 steps of 16 dims: unit kk / 4, +32 B within it
          tc_mma(ts, sw128_desc(q0 + (kk >> 2) * AT_UNIT) + 2 * (kk & 3), sw128_desc(kt + (kk >> 2) * 8192) + 2 * (kk & 3),
                 AT_IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(&k_empty[s]);
        tc_commit(&s_full[s]);
        if (i > 0) ok = mma2(i - 1);
      }
      if (ok && n_blocks > 0) mma2(n_blocks - 1);
    }
    __syncwarp();
  } else if (warp < 4) {
    // warps 2-3: idle (the P V product reads V as loaded, MN-major)
  } else {
    // ---------------- softmax (one thread per row, TMEM lanes 0-63) and epilogue ----------------
    const int r = threadIdx.x - 128;  // row of the MMA tile: head hl = r / 16, token tr = r % 16
    const int hl = r >> 4, tr = r & 15;
    const bool real = hl < G;
    const int lim = real ? s_lim[tr] : 0;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n_blocks && ok; ++i) {
      const int s = i & 1;
      if (!mbar_wait(&s_full[s], (i >> 1) & 1, 328, a.err)) { ok = false; break; }
      tc_fence_after();
      float sv[64];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tc_ld16(tmem + lane_base + (uint32_t)(s * 64 + q4 * 16), sv + q4 * 16);
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      const int kb = k_begin + i * AT_KB;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int key = kb + c;
        sv[c] = (key < lim && key < k_end) ? sv[c] * a.scale_log2 : -INFINITY;
        mx = fmaxf(mx, sv[c]);
      }
      // P buffer i & 1 is free once the P V product of block i - 2 has read it
      if (i > 1 && !mbar_wait(&p_free[i & 1], ((i - 2) >> 1) & 1, 329, a.err)) { ok = false; break; }
      // tcgen05.ld / st are warp-collective: the warp rescales O together whenever any of
      // its rows needs it, rows that do not with factor 1 (exact)
      const bool resc = mx > m_used + AT_RESCALE || (m_used == -INFINITY && mx > -INFINITY);
      const float f = !resc ? 1.f : (m_used == -INFINITY ? 0.f : exp2f(m_used - mx));
      if (resc) {
        l *= f;
        m_used = mx;
      }
      if (i > 0 && __any_sync(0xffffffffu, resc)) {
        // O must be complete up to block i - 1 before it is rescaled
        if (!mbar_wait(&p_free[(i - 1) & 1], ((i - 1) >> 1) & 1, 330, a.err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) {
          float ov[16];
          tc_ld16(t_o + lane_base + (uint32_t)(q8 * 16), ov);
#pragma unroll
          for (int e = 0; e < 16; ++e) ov[e] *= f;
          tc_st16(t_o + lane_base + (uint32_t)(q8 * 16), ov);
        }
        tc_fence_before();
      }
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      float ps = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float p0 = exp2f(sv[c8 * 8 + 2 * u] - mu), p1 = exp2f(sv[c8 * 8 + 2 * u + 1] - mu);
          ps += p0 + p1;
          const float h0 = round_bf16(p0), h1 = round_bf16(p1);
          hi[u] = pack_bf16x2(h0, h1);
          lo[u] = pack_bf16x2(p0 - h0, p1 - h1);
        }
        unsigned char* pb = smem + AT_OFF_P + (i & 1) * 2 * AT_UNIT;
        *reinterpret_cast<uint4*>(pb + sw_off(r, c8)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(pb + AT_UNIT + sw_off(r, c8)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      l += ps;
      fence_proxy_async_smem();
      mbar_arrive(&p_full[i & 1]);
    }
    // epilogue: O of this row once the last P V product completed (every thread of the warp
    // loads its TMEM lane -- the loads are warp-collective -- and valid rows store)
    if (__all_sync(0xffffffffu, ok) &&
        mbar_wait(&p_free[(n_blocks - 1) & 1], ((n_blocks - 1) >> 1) & 1, 329, a.err)) {
      tc_fence_after();
      const bool store = real && lim > k_begin && m0 + tr < a.M;
      const int m = m0 + tr, h = kvh * G + hl;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = a.out + (long long)m * a.ldo + (long long)h * AT_HD;
      const long long base = ((long long)chunk * a.M + m) * a.Hq + h;
      float* po = a.part_o + base * AT_HD;
#pragma unroll
      for (int q8 = 0; q8 < 8; ++q8) {
        float ov[16];
        tc_ld16(t_o + lane_base + (uint32_t)(q8 * 16), ov);
        if (!store) continue;
        if (a.direct) {
          uint4 w0, w1;
          w0.x = pack_bf16x2(ov[0] * inv, ov[1] * inv);
          w0.y = pack_bf16x2(ov[2] * inv, ov[3] * inv);
          w0.z = pack_bf16x2(ov[4] * inv, ov[5] * inv);
          w0.w = pack_bf16x2(ov[6] * inv, ov[7] * inv);
          w1.x = pack_bf16x2(ov[8] * inv, ov[9] * inv);
          w1.y = pack_bf16x2(ov[10] * inv, ov[11] * inv);
          w1.z = pack_bf16x2(ov[12] * inv, ov[13] * inv);
          w1.w = pack_bf16x2(ov[14] * inv, ov[15] * inv);
          *reinterpret_cast<uint4*>(dst + q8 * 16) = w0;
          *reinterpret_cast<uint4*>(dst + q8 * 16 + 8) = w1;
        } else {
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4)
            *reinterpret_cast<float4*>(po + q8 * 16 + e4 * 4) =
                make_float4(ov[4 * e4], ov[4 * e4 + 1], ov[4 * e4 + 2], ov[4 * e4 + 3]);
        }
      }
      if (store && !a.direct) a.part_ml[base] = make_float2(m_used, l);
      tc_fence_before();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "n"(AT_TMEM_COLS));
  }
}

// ---- host: 3-D tensor maps over the caches (dims x key rows x planes) ----------------
struct Map3Key {
  const void* base;
  uint64_t rows, planes, plane_stride;
  bool operator==(const Map3Key& o) const {
    return base == o.base && rows == o.rows && planes == o.planes && plane_stride == o.plane_stride;
  }
};
struct Map3Hash {
  size_t operator()(const Map3Key& k) const {
    return std::hash<const void*>()(k.base) ^ (std::hash<uint64_t>()(k.rows) * 31) ^ (k.plane_stride * 131);
  }
};
static std::mutex g_map3_mu;
static std::unordered_map<Map3Key, CUtensorMap, Map3Hash>* g_maps3 = nullptr;
static PFN_cuTensorMapEncodeTiled g_encode3 = nullptr;

// [planes][rows][128] bf16 with planes plane_stride elements apart, box 64 x 64 x 1, 128-byte swizzle
static bool tensor_map_kv(const void* base, uint64_t rows, uint64_t planes, uint64_t plane_stride, CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_map3_mu);
  if (!g_maps3) g_maps3 = new std::unordered_map<Map3Key, CUtensorMap, Map3Hash>();
  Map3Key key{base, rows, planes, plane_stride};
  auto it = g_maps3->find(key);
  if (it != g_maps3->end()) {
    *out = it->second;
    return true;
  }
  if (!g_encode3) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      set_error("cuTensorMapEncodeTiled is not available from the driver");
      return false;
    }
    g_encode3 = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  CUtensorMap map;
  cuuint64_t dims[3] = {AT_HD, rows, planes};
  cuuint64_t strides[2] = {AT_HD * 2, plane_stride * 2};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode3(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D cache map) failed (%d)", (int)r);
    return false;
  }
  if (g_maps3->size() > 4096) g_maps3->clear();
  g_maps3->emplace(key, map);
  *out = map;
  return true;
}

// Whether the tensor-core form takes this call: opt in with DFLASH_B200_ATTN_TC=1 (a
// process-wide choice, so every launch of a session agrees). Off by default: on B200 it
// measured slower than the mma.sync form at both verify shapes (single stream 24.2 against
// 19.2 us, 64 sequences 324 against 236 us): two softmax warps per CTA and one CTA per SM
// leave the exponentials on the critical path of every 64-key block.
bool attention_tc_ok(int hd, int G, bool gated, bool fused) {
  static const bool enabled = [] {
    const char* e = getenv("DFLASH_B200_ATTN_TC");
    return e && e[0] == '1';
  }();
  return enabled && hd == AT_HD && G >= 1 && G * 16 <= 128 && !gated && !fused;
}

// Launches the tensor-core chunk kernel. The caches are dense: [seq][Hkv][cap][128] (head
// stride cap * 128, sequence stride Hkv * head stride) or, with a page table, pages
// [page][Hkv][page_size][128].
int launch_attention_tc(const void* q, const void* k_cache, const void* v_cache, long long seq_stride,
                        long long head_stride, const int* pos, const int* row_seq, const int* kv_len,
                        const int* page_table, long long pt_stride, int page_shift, int M, int Hq, int Hkv,
                        int causal, float scale_log2, int n_chunks, int segs, int key_chunk, float* part_o,
                        float2* part_ml, void* out, long long ldo, int n_tiles, int* err, cudaStream_t st) {
  if (head_stride % AT_HD || seq_stride != (long long)Hkv * head_stride) {
    set_error("dfl_attention: the tensor-core form needs dense caches (sequence stride = Hkv x head stride)");
    return DFL_ERR_UNSUPPORTED;
  }
  const uint64_t rows = (uint64_t)(head_stride / AT_HD);  // cap, or the page size
  // planes up to the end of the allocation holding the caches (only real ones are read)
  uint64_t planes = 0;
  {
    typedef CUresult (*RangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
    static RangeFn range_fn = nullptr;
    if (!range_fn) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult qr;
      if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &qr) == cudaSuccess &&
          qr == cudaDriverEntryPointSuccess)
        range_fn = reinterpret_cast<RangeFn>(fn);
    }
    for (const void* p : {k_cache, v_cache}) {
      CUdeviceptr b = 0;
      size_t sz = 0;
      if (!range_fn || range_fn(&b, &sz, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) {
        set_error("dfl_attention: cannot find the allocation of the K/V caches");
        return DFL_ERR_UNSUPPORTED;
      }
      const uint64_t n = (uint64_t)(b + sz - reinterpret_cast<CUdeviceptr>(p)) / ((uint64_t)head_stride * 2);
      planes = planes == 0 ? n : (n < planes ? n : planes);
    }
    if (planes == 0) {
      set_error("dfl_attention: K/V caches smaller than one head plane");
      return DFL_ERR_UNSUPPORTED;
    }
  }
  AttnTcMaps maps;
  if (!tensor_map_kv(k_cache, rows, planes, (uint64_t)head_stride, &maps.k) ||
      !tensor_map_kv(v_cache, rows, planes, (uint64_t)head_stride, &maps.v))
    return DFL_ERR_CUDA;
  AttnTcArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.pos = pos;
  a.row_seq = row_seq;
  a.kv_len = kv_len;
  a.page_table = page_table;
  a.pt_stride = pt_stride;
  a.page_shift = page_shift;
  a.planes_per_seq = Hkv;
  a.part_o = part_o;
  a.part_ml = part_ml;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.M = M;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.causal = causal;
  a.n_chunks = n_chunks;
  a.segs = segs;
  a.key_chunk = key_chunk;
  a.direct = n_chunks == 1;
  a.scale_log2 = scale_log2;
  a.err = err;
  static bool init[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !init[dev]) {
    if (cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM) != cudaSuccess) {
      set_error("dfl_attention: cannot opt in to %d bytes of shared memory", AT_SMEM);
      return DFL_ERR_UNSUPPORTED;
    }
    init[dev] = true;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_chunks, Hkv, n_tiles * segs);
  cfg.blockDim = dim3(AT_THREADS);
  cfg.dynamicSmemBytes = AT_SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_tc_kernel, maps, a);
  if (e != cudaSuccess) {
    set_error("dfl_attention: tensor-core kernel launch failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

}  // namespace dfl
