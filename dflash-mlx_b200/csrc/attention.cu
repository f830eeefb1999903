// Grouped-query attention of a block of query tokens against a per-sequence KV cache.
//
// Replaces mx.fast.scaled_dot_product_attention as called by the verify forward
// (mlx-lm qwen3 Attention, mask "causal" from qwen3.create_attention_mask,
// adapters.py:620) and by the DFlash draft (draft.py:149-157, mask none or causal).
//
//   o[m, h] = softmax_j( scale * q[m, h] . K[kvh(h), j] ) V[kvh(h), j],   j < lim(m)
//   lim(m)  = pos[m] + 1           (causal: the key at the query's own position is the last one)
//           = kv_len[seq(m)]       (non-causal)
//
// Layout: q [M][Hq][hd] bf16, caches [seq][Hkv][cap][hd] bf16 (slot == position).
// Work split: one CTA per (key chunk of key_chunk keys, kv head, 16-token
// tile, sequence segment of the tile); the rows of a tile that belong to the
// segment's sequence are the CTA's rows (a batched verify block of fewer than
// 16 rows per sequence puts several sequences in one tile, each read from its own
// cache); warp w of the CTA owns q head kvh*G + w for the 16 tokens, so the G
// query heads sharing a kv head read each K/V tile once. Chunks are fixed
// absolute key ranges and are merged in chunk order by a second kernel, so a
// query row's result does not depend on the other rows or on keys it cannot
// see (spec-verify rows and plain-decode rows agree bit for bit). The chunk size
// is the caller's (DFL_ATTN_CHUNK by default): small chunks spread one sequence
// over many SMs, large ones cut the partial-result traffic of batched verify.
// When one chunk covers every row's keys the chunk kernel normalises and writes
// the output itself (the merge of a single chunk is the identity) and no merge
// kernel runs. K/V stream through a 3-stage cp.async ring (2 stages at head_dim 256).
// (A variant that merged the chunks inside the chunk kernel, one thread-block cluster per
// tile and kv head reading the peers' partials over distributed shared memory, measured
// slower on B200 at both the single-stream and the 64-sequence shapes and was removed.)
#include "common.cuh"
#include "tma_util.cuh"

namespace dfl {

constexpr int ATT_SITE_SEGMENTS = 301;  // a tile held more sequences than the launch's segments

constexpr int ATT_KB = 64;              // keys per shared-memory sub-block

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  long long seq_stride, head_stride;
  const int* pos;
  const int* row_seq;
  const int* kv_len;
  float* part_o;   // [chunks][M][Hq][hd]
  float2* part_ml; // [chunks][M][Hq]
  __nv_bfloat16* out;
  long long ldo;
  const __nv_bfloat16* gate;  // nullable: out *= sigmoid(gate) (Qwen3.5 gated attention)
  long long ldg;
  int gate_hs;  // elements between consecutive heads' gates in a row
  int M, Hq, Hkv, G, causal, n_chunks;
  int segs;          // sequence segments per 16-row tile (grid z = tiles * segs)
  int key_chunk;     // keys per chunk (multiple of 64)
  int direct;        // one chunk: the chunk kernel writes the normalised output
  int* err;          // device error record
  float scale_log2;  // softmax scale * log2(e)
  // fused q/k head norm + RoPE + cache append (head_dim 128, full rotary): q and the new
  // keys / values come from the raw projection rows instead of q and a prior append
  const __nv_bfloat16* qkv;  // nullable: [M][(Hq + 2 Hkv) * 128] rows
  long long ldqkv;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* inv_freq;  // [64]
  float eps;
  __nv_bfloat16* k_new;   // the caches, written at the new rows' positions
  __nv_bfloat16* v_new;
  // paged caches: [page][Hkv][page_size][hd] with seq_stride = the page stride; position p
  // of sequence s is row p % page_size of page page_table[s * pt_stride + p / page_size]
  const int* page_table;
  long long pt_stride;
  int page_shift;
};

// element offset, from the cache base plus the kv head, of the 64-key block starting at
// key kb (a block never straddles a page: page sizes are multiples of 64)
__device__ __forceinline__ long long kv_block_offset(const AttnArgs& a, int seq, int kb, int hd) {
  if (!a.page_table) return (long long)seq * a.seq_stride + (long long)kb * hd;
  const long long page = a.page_table[seq * a.pt_stride + (kb >> a.page_shift)];
  return page * a.seq_stride + (long long)(kb & ((1 << a.page_shift) - 1)) * hd;
}

// One 128-wide head row held 4 values per lane (element lane + 32 j): RMSNorm with weight
// nw, then the rotary embedding with the row's (cos, sin) table cs[64] -- the arithmetic of
// qkv_rope_append_kernel (same summation order, same pinned roundings, the same sincosf
// values), so both paths give the same bits.
__device__ __forceinline__ void norm_rope_row128(float (&x)[4], const __nv_bfloat16* nw, const float2* cs,
                                                 float eps, int lane) {
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss = sq_acc(ss, x[j]);
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / 128.f + eps);
  float y[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) y[j] = round_bf16(bf2f(nw[lane + 32 * j]) * (x[j] * inv));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = cs[lane + 32 * (j & 1)];
    x[j] = rope_rot(y[j], y[j ^ 2], t.x, t.y, j < 2);
  }
}

template <int HD>
__device__ __forceinline__ int att_swz(int row, int c) {
  return row * HD + ((c ^ (row & 7)) << 3);
}

__device__ __forceinline__ int row_limit(const AttnArgs& a, int m) {
  if (m >= a.M) return 0;
  const int p = a.pos[m];
  if (p < 0) return 0;
  if (a.causal) return p + 1;
  const int s = a.row_seq ? a.row_seq[m] : 0;
  return a.kv_len[s];
}

// K/V ring depth: 3 stages for long chunks at head_dim <= 128; 2 for short chunks
// (a 128-key chunk is two blocks: a deeper ring only costs shared memory that the
// next kernel's prologue could use) and for head_dim 256 (shared memory)
template <int HD, int ST>
__global__ void __launch_bounds__(256) attn_chunk_kernel(AttnArgs a) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  constexpr int NC = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [G][16][HD]
  __nv_bfloat16* sK = sQ + a.G * 16 * HD;                           // [ST][64][HD]
  __nv_bfloat16* sV = sK + ST * ATT_KB * HD;                         // [ST][64][HD]

  const int chunk = blockIdx.x, kvh = blockIdx.y, tile = blockIdx.z / a.segs, seg = blockIdx.z % a.segs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nthr = blockDim.x;
  const int m0 = tile * 16;

  __shared__ int s_lim[16];
  __shared__ int s_seq;
  if (threadIdx.x < 32) {
    // warp 0: the tile's rows (lane r < 16), the first row of each sequence in the tile,
    // and this CTA's sequence = the seg-th of them in row order
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
      for (int k = 0; k < seg; ++k) msk &= msk - 1;  // drop the seg lowest first-rows
      row = __ffs(msk) - 1;
    }
    const int chosen = __shfl_sync(0xffffffffu, sq, row < 0 ? 0 : row);
    if (r == 0) {
      if (seg == 0 && n > a.segs && chunk == 0 && kvh == 0 && a.err) atomicCAS(a.err, 0, ATT_SITE_SEGMENTS);
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

  const __nv_bfloat16* Kb = a.k_cache + kvh * a.head_stride;
  const __nv_bfloat16* Vb = a.v_cache + kvh * a.head_stride;

  if constexpr (HD == 128) {
    if (a.qkv) {
      // fused append: this CTA's new rows whose position falls in its key range get their
      // key (norm + RoPE) and value written to the cache here -- no other CTA reads them,
      // since every row of a sequence is in this tile and every CTA reads only its own
      // key range -- then the Q tile is normalised and rotated from the projection rows
      const int Hq = a.Hq;
      // (cos, sin) of every row's position and frequency, once per CTA, in the K ring
      // (idle until the ring prologue below, which follows the barrier after this block)
      float2(*s_cs)[64] = reinterpret_cast<float2(*)[64]>(sK);
      for (int idx = threadIdx.x; idx < 16 * 64; idx += nthr) {
        const int r = idx >> 6, f = idx & 63;
        const int p = s_lim[r] > 0 ? a.pos[m0 + r] : 0;
        float sn, cs;
        sincosf(rope_angle(p, a.inv_freq[f]), &sn, &cs);
        s_cs[r][f] = make_float2(cs, sn);
      }
      __syncthreads();
      for (int r = warp; r < 16; r += a.G) {
        const int m = m0 + r;
        if (s_lim[r] <= 0) continue;
        const int p = a.pos[m];
        if (p < k_begin || p >= k_end) continue;
        const __nv_bfloat16* row = a.qkv + (long long)m * a.ldqkv;
        const __nv_bfloat16* ks = row + (long long)(Hq + kvh) * 128;
        const __nv_bfloat16* vs = row + (long long)(Hq + a.Hkv + kvh) * 128;
        float x[4];
        __nv_bfloat16 vv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          x[j] = bf2f(ks[lane + 32 * j]);
          vv[j] = vs[lane + 32 * j];
        }
        norm_rope_row128(x, a.k_norm, s_cs[r], a.eps, lane);
        const long long off = kv_block_offset(a, s_seq, p & ~(ATT_KB - 1), 128) + kvh * a.head_stride +
                              (long long)(p & (ATT_KB - 1)) * 128;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          a.k_new[off + lane + 32 * j] = f2bf(x[j]);
          a.v_new[off + lane + 32 * j] = vv[j];
        }
      }
      // Q: warp w holds head kvh * G + w; four rows' loads in flight at a time
      const int hq = kvh * a.G + warp;
      __nv_bfloat16* myq = sQ + warp * 16 * HD;
#pragma unroll 1
      for (int r0 = 0; r0 < 16; r0 += 4) {
        float x[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int m = m0 + r0 + u;
          const bool ok = s_lim[r0 + u] > 0;
          const __nv_bfloat16* qs = a.qkv + (long long)(ok ? m : 0) * a.ldqkv + (long long)hq * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) x[u][j] = ok ? bf2f(qs[lane + 32 * j]) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = r0 + u;
          if (s_lim[r] > 0) norm_rope_row128(x[u], a.q_norm, s_cs[r], a.eps, lane);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int i = lane + 32 * j;
            myq[att_swz<HD>(r, i >> 3) + (i & 7)] = s_lim[r] > 0 ? f2bf(x[u][j]) : __float2bfloat16(0.f);
          }
        }
      }
      __threadfence();  // the appended rows reach L2 before this CTA's cp.async reads them
      __syncthreads();
    }
  }
  // Q tile: rows are (head-in-group, token)
  for (int idx = threadIdx.x; idx < (a.qkv ? 0 : a.G * 16 * NC); idx += nthr) {
    const int c = idx % NC;
    const int rr = idx / NC;  // hg*16 + r
    const int hg = rr / 16, r = rr % 16;
    const int m = m0 + r;
    const bool ok = m < a.M && s_lim[r] > 0;
    const __nv_bfloat16* src = a.q + ((long long)(ok ? m : 0) * a.Hq + kvh * a.G + hg) * HD + c * 8;
    cp_async16(smem_u32(sQ + hg * 16 * HD + att_swz<HD>(r, c)), src, ok ? 16 : 0);
  }
  auto load_kv = [&](int buf, int kb) {
    const long long boff = kv_block_offset(a, s_seq, kb, HD);
    for (int idx = threadIdx.x; idx < ATT_KB * NC; idx += nthr) {
      const int c = idx % NC, r = idx / NC;
      const int key = kb + r;
      const bool ok = key < k_end;
      const long long off = boff + (long long)(ok ? r : 0) * HD + c * 8;
      cp_async16(smem_u32(sK + buf * ATT_KB * HD + att_swz<HD>(r, c)), Kb + off, ok ? 16 : 0);
      cp_async16(smem_u32(sV + buf * ATT_KB * HD + att_swz<HD>(r, c)), Vb + off, ok ? 16 : 0);
    }
  };
  // ring prologue: Q and the first ST - 1 key blocks
#pragma unroll
  for (int st = 0; st < ST - 1; ++st) {
    if (k_begin + st * ATT_KB < k_end) load_kv(st, k_begin + st * ATT_KB);
    cp_async_commit();
  }

  const int g = lane >> 2, t = lane & 3;
  const int lim0 = s_lim[g], lim1 = s_lim[g + 8];
  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};
  const __nv_bfloat16* myQ = sQ + warp * 16 * HD;

  int buf = 0;
  for (int kb = k_begin; kb < k_end; kb += ATT_KB) {
    cp_async_wait<ST - 2>();
    __syncthreads();  // block kb landed for every thread; the stage refilled below was consumed last iteration
    {
      const int nb = kb + (ST - 1) * ATT_KB;
      const int nbuf = buf == 0 ? ST - 1 : buf - 1;
      if (nb < k_end) load_kv(nbuf, nb);
      cp_async_commit();
    }
    const __nv_bfloat16* tK = sK + buf * ATT_KB * HD;
    const __nv_bfloat16* tV = sV + buf * ATT_KB * HD;

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t af[4];
      {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = 2 * ks + (lane >> 4);
        ldmatrix_x4(smem_u32(myQ + att_swz<HD>(row, c)), af[0], af[1], af[2], af[3]);
      }
#pragma unroll
      for (int nb = 0; nb < 4; ++nb) {
        const int row = nb * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = 2 * ks + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_u32(tK + att_swz<HD>(row, c)), b0, b1, b2, b3);
        mma_bf16_16816(s[2 * nb], af, b0, b1);
        mma_bf16_16816(s[2 * nb + 1], af, b2, b3);
      }
    }
    // mask + online softmax (log2 domain)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int key = kb + j * 8 + 2 * t;
      s[j][0] = key < lim0 ? s[j][0] * a.scale_log2 : -INFINITY;
      s[j][1] = key + 1 < lim0 ? s[j][1] * a.scale_log2 : -INFINITY;
      s[j][2] = key < lim1 ? s[j][2] * a.scale_log2 : -INFINITY;
      s[j][3] = key + 1 < lim1 ? s[j][3] * a.scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(mrow[0], mx0), mn1 = fmaxf(mrow[1], mx1);
    const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(mrow[0] - mu0), al1 = exp2f(mrow[1] - mu1);
    mrow[0] = mn0;
    mrow[1] = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = exp2f(s[j][0] - mu0);
      s[j][1] = exp2f(s[j][1] - mu0);
      s[j][2] = exp2f(s[j][2] - mu1);
      s[j][3] = exp2f(s[j][3] - mu1);
      ps0 += s[j][0] + s[j][1];
      ps1 += s[j][2] + s[j][3];
    }
    lrow[0] = lrow[0] * al0 + ps0;
    lrow[1] = lrow[1] * al1 + ps1;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      o[j][0] *= al0;
      o[j][1] *= al0;
      o[j][2] *= al1;
      o[j][3] *= al1;
    }
    // O += P V, with P split into bf16 high and low parts (P = hi + lo to about 16
    // significant bits): the probabilities keep near-fp32 precision, as the reference's
    // fp32 softmax weights do, instead of a single bf16 rounding of each weight
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pf[4], pl[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float x0 = s[2 * kk + (u >> 1)][2 * (u & 1)], x1 = s[2 * kk + (u >> 1)][2 * (u & 1) + 1];
        const float h0 = round_bf16(x0), h1 = round_bf16(x1);
        pf[u] = pack_bf16x2(h0, h1);
        pl[u] = pack_bf16x2(x0 - h0, x1 - h1);
      }
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        const int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = 2 * dp + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(smem_u32(tV + att_swz<HD>(row, c)), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * dp], pf, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pf, b2, b3);
        mma_bf16_16816(o[2 * dp], pl, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pl, b2, b3);
      }
    }
    buf = buf == ST - 1 ? 0 : buf + 1;
  }
  cp_async_wait<0>();

  lrow[0] += __shfl_xor_sync(0xffffffffu, lrow[0], 1);
  lrow[0] += __shfl_xor_sync(0xffffffffu, lrow[0], 2);
  lrow[1] += __shfl_xor_sync(0xffffffffu, lrow[1], 1);
  lrow[1] += __shfl_xor_sync(0xffffffffu, lrow[1], 2);

  const int h = kvh * a.G + warp;
  if (a.direct) {
    // single chunk: out = o / l (the merge of one chunk is the identity)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = g + half * 8;
      const int m = m0 + r;
      if (m >= a.M || s_lim[r] <= 0) continue;
      const float den = lrow[half];
      const float inv = den > 0.f ? 1.f / den : 0.f;
      __nv_bfloat16* dst = a.out + (long long)m * a.ldo + (long long)h * HD;
      const __nv_bfloat16* gr = a.gate ? a.gate + (long long)m * a.ldg + (long long)h * a.gate_hs : nullptr;
#pragma unroll
      for (int j = 0; j < HD / 8; ++j) {
        const int d = j * 8 + 2 * t;
        float y0 = o[j][2 * half] * inv, y1 = o[j][2 * half + 1] * inv;
        if (gr) {
          y0 = round_bf16(y0) * round_bf16(1.f / (1.f + __expf(-bf2f(gr[d]))));
          y1 = round_bf16(y1) * round_bf16(1.f / (1.f + __expf(-bf2f(gr[d + 1]))));
        }
        *reinterpret_cast<uint32_t*>(dst + d) = pack_bf16x2(y0, y1);
      }
    }
    return;
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = g + half * 8;
    const int m = m0 + r;
    if (m >= a.M || s_lim[r] <= k_begin) continue;
    const long long base = ((long long)chunk * a.M + m) * a.Hq + h;
    float* po = a.part_o + base * HD;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      *reinterpret_cast<float2*>(po + j * 8 + 2 * t) = make_float2(o[j][2 * half], o[j][2 * half + 1]);
    }
    if (t == 0) a.part_ml[base] = make_float2(mrow[half], lrow[half]);
  }
}

// Merge the chunk partials of one (row, head) in chunk order. One warp per
// (row, head): lane c holds chunk c's (max, sum) so the global max and the
// denominator are warp reductions; the output accumulates chunk by chunk in
// order, eight chunks' loads in flight at a time (four at head_dim 256). The first
// 32 chunks' (max, sum) and the first eight chunks' outputs are loaded together with
// the row's key range, before it is known which of them the row uses.
template <int HD>
__global__ void attn_combine_kernel(AttnArgs a) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (item >= (long long)a.M * a.Hq) return;
  const int m = (int)(item / a.Hq), h = (int)(item % a.Hq);
  constexpr int PER = HD / 32;
  constexpr int FL = HD <= 128 ? 8 : 4;  // chunks' loads in flight
  const long long cstride = (long long)a.M * a.Hq;  // between one chunk's partials and the next's
  const float2* ml_row = a.part_ml + (long long)m * a.Hq + h;
  const float* po_row = a.part_o + ((long long)m * a.Hq + h) * HD;
  // Loads that do not depend on the row's key range go out with the range's own loads:
  // the first 32 chunks' (max, sum) and the first FL chunks' partial outputs (only the
  // row's own chunks are used below).
  const int pre_ml = min(32, a.n_chunks), pre_o = min(FL, a.n_chunks);
  const float2 ml0 = lane < pre_ml ? ml_row[lane * cstride] : make_float2(-INFINITY, 0.f);
  float v0[FL][PER];
#pragma unroll
  for (int u = 0; u < FL; ++u)
#pragma unroll
    for (int i = 0; i < PER; ++i) v0[u][i] = u < pre_o ? po_row[u * cstride * HD + lane + 32 * i] : 0.f;
  const int lim = row_limit(a, m);
  if (lim <= 0) return;
  const int nch = min((lim + a.key_chunk - 1) / a.key_chunk, a.n_chunks);
  float acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.f;
  float den = 0.f;
  // global max over the row's chunks
  float mmax = lane < nch ? ml0.x : -INFINITY;
  for (int c = lane + 32; c < nch; c += 32) mmax = fmaxf(mmax, ml_row[c * cstride].x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, o));
  const float mu = mmax == -INFINITY ? 0.f : mmax;
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const int c = c0 + lane;
    const float2 ml = c >= nch ? make_float2(-INFINITY, 0.f) : (c0 == 0 ? ml0 : ml_row[c * cstride]);
    const float w = c < nch ? exp2f(ml.x - mu) : 0.f;
    float dl = w * ml.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dl += __shfl_xor_sync(0xffffffffu, dl, o);
    den += dl;
    const int n = min(32, nch - c0);
    int j = 0;
    if (c0 == 0) {  // the prefetched chunks, in order
#pragma unroll
      for (int u = 0; u < FL; ++u)
        if (u < n) {
          const float wj = __shfl_sync(0xffffffffu, w, u);
#pragma unroll
          for (int i = 0; i < PER; ++i) acc[i] += wj * v0[u][i];
        }
      j = min(FL, n);
    }
    for (; j + FL <= n; j += FL) {
      float v[FL][PER];
      float wj[FL];
#pragma unroll
      for (int u = 0; u < FL; ++u) {
        wj[u] = __shfl_sync(0xffffffffu, w, j + u);
        const float* po = po_row + (long long)(c0 + j + u) * cstride * HD;
#pragma unroll
        for (int i = 0; i < PER; ++i) v[u][i] = po[lane + 32 * i];
      }
#pragma unroll
      for (int u = 0; u < FL; ++u)
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[i] += wj[u] * v[u][i];
    }
    for (; j < n; ++j) {
      const float wj = __shfl_sync(0xffffffffu, w, j);
      const float* po = po_row + (long long)(c0 + j) * cstride * HD;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[i] += wj * po[lane + 32 * i];
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  __nv_bfloat16* dst = a.out + (long long)m * a.ldo + (long long)h * HD;
  if (a.gate) {
    // o_proj(attn * sigmoid(gate)), custom_qwen35_model.py:193
    const __nv_bfloat16* gr = a.gate + (long long)m * a.ldg + (long long)h * a.gate_hs;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const float gt = bf2f(gr[lane + 32 * i]);
      dst[lane + 32 * i] = f2bf(round_bf16(acc[i] * inv) * round_bf16(1.f / (1.f + __expf(-gt))));
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = f2bf(acc[i] * inv);
  }
}

// the ordered merge of the chunk partials (one warp per row and head)
template <int HD>
static int launch_combine(const AttnArgs& a, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  const long long items = (long long)a.M * a.Hq;
  cfg.gridDim = dim3((unsigned)((items + 7) / 8));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_combine_kernel<HD>, a);
  if (e != cudaSuccess) {
    set_error("dfl_attention: combine launch failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

// tensor-core form (attention_tc.cu)
bool attention_tc_ok(int hd, int G, bool gated, bool fused);
int launch_attention_tc(const void* q, const void* k_cache, const void* v_cache, long long seq_stride,
                        long long head_stride, const int* pos, const int* row_seq, const int* kv_len,
                        const int* page_table, long long pt_stride, int page_shift, int M, int Hq, int Hkv,
                        int causal, float scale_log2, int n_chunks, int segs, int key_chunk, float* part_o,
                        float2* part_ml, void* out, long long ldo, int n_tiles, int* err, cudaStream_t st);

template <int HD, int ST>
static int launch_attn(AttnArgs a, int n_tiles, cudaStream_t st) {
  const size_t smem = (size_t)(a.G * 16 * HD + 2 * ST * ATT_KB * HD) * 2;
  // opt in once per device to the whole per-block shared memory: the SM then keeps its
  // largest shared-memory carveout, which the GEMMs before and after this kernel use, so
  // their CTAs can stay co-resident with it (programmatic dependent launch overlap)
  static bool opted[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !opted[dev]) {
    cudaFuncAttributes fa;
    int optin = 0;
    if (cudaFuncGetAttributes(&fa, attn_chunk_kernel<HD, ST>) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncSetAttribute(attn_chunk_kernel<HD, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)fa.sharedSizeBytes) != cudaSuccess) {
      set_error("dfl_attention: cannot opt in to the per-block shared memory");
      return DFL_ERR_UNSUPPORTED;
    }
    opted[dev] = true;
  }
  if (smem > 227 * 1024) {
    set_error("dfl_attention: %zu bytes of shared memory needed", smem);
    return DFL_ERR_UNSUPPORTED;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_chunks, a.Hkv, n_tiles * a.segs);
  cfg.blockDim = dim3(32 * a.G);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attn_chunk_kernel<HD, ST>, a);
  if (e != cudaSuccess) {
    set_error("dfl_attention: chunk kernel launch failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  if (a.direct) return DFL_OK;
  return launch_combine<HD>(a, st);
}

}  // namespace dfl

using namespace dfl;

static int resolve_key_chunk(int key_chunk) { return key_chunk > 0 ? key_chunk : DFL_ATTN_CHUNK; }

extern "C" size_t dfl_attention_workspace_bytes(int M, int Hq, int hd, int max_kv, int key_chunk) {
  if (M <= 0 || max_kv <= 0) return 0;
  key_chunk = resolve_key_chunk(key_chunk);
  if (key_chunk % 64) return 0;
  const size_t nch = (size_t)(max_kv + key_chunk - 1) / key_chunk;
  if (nch <= 1) return 0;  // single chunk: no partials
  const size_t o = nch * M * Hq * hd * sizeof(float);
  const size_t ml = nch * M * Hq * sizeof(float2);
  return ((o + 255) & ~(size_t)255) + ml;
}

namespace {
struct FusedQkv {
  const void* qkv;
  int64_t ldqkv;
  const void* q_norm;
  const void* k_norm;
  const float* inv_freq;
  float eps;
};
}  // namespace

static int attention_impl(const void* q, const void* k_cache, const void* v_cache, int64_t seq_stride,
                          int64_t head_stride, const int32_t* pos, const int32_t* row_seq, const int32_t* kv_len,
                          int seq_rows, int M, int Hq, int Hkv, int hd, int causal, float scale, int max_kv,
                          int key_chunk, void* out, int64_t ldo, const void* gate, int64_t ldg, int gate_head_stride,
                          void* workspace, size_t workspace_bytes, void* stream, const FusedQkv* fq,
                          const int32_t* page_table = nullptr, int64_t pt_stride = 0, int page_size = 0) {
  if (M == 0) return DFL_OK;
  if ((!q && !fq) || !k_cache || !v_cache || !pos || !out || (!causal && !kv_len) || M < 0 || Hkv <= 0 ||
      Hq % Hkv) {
    set_error("dfl_attention: bad arguments");
    return DFL_ERR_INVALID;
  }
  const int G = Hq / Hkv;
  if (G < 1 || G > 8) {
    set_error("dfl_attention: query heads per kv head must be 1..8 (got %d)", G);
    return DFL_ERR_UNSUPPORTED;
  }
  if (max_kv <= 0) {
    set_error("dfl_attention: max_kv must be positive");
    return DFL_ERR_INVALID;
  }
  key_chunk = resolve_key_chunk(key_chunk);
  if (key_chunk % 64) {
    set_error("dfl_attention: key_chunk %d must be a multiple of 64", key_chunk);
    return DFL_ERR_INVALID;
  }
  const size_t need = dfl_attention_workspace_bytes(M, Hq, hd, max_kv, key_chunk);
  if (need && (!workspace || workspace_bytes < need)) {
    set_error("dfl_attention: workspace too small (%zu < %zu)", workspace_bytes, need);
    return DFL_ERR_WORKSPACE;
  }
  AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
  a.seq_stride = seq_stride;
  a.head_stride = head_stride;
  a.pos = pos;
  a.row_seq = row_seq;
  a.kv_len = kv_len;
  a.key_chunk = key_chunk;
  a.n_chunks = (max_kv + key_chunk - 1) / key_chunk;
  a.direct = a.n_chunks == 1;
  const size_t o_bytes = (size_t)a.n_chunks * M * Hq * hd * sizeof(float);
  a.part_o = static_cast<float*>(workspace);
  a.part_ml = reinterpret_cast<float2*>(static_cast<char*>(workspace) + ((o_bytes + 255) & ~(size_t)255));
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.ldg = ldg;
  a.gate_hs = gate_head_stride > 0 ? gate_head_stride : hd;
  a.M = M;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = G;
  a.causal = causal;
  a.scale_log2 = scale * 1.4426950408889634f;
  const int n_tiles = (M + 15) / 16;
  const bool deep = key_chunk > 2 * ATT_KB;
  // sequences a 16-row tile can hold: one without row_seq or when sequences are
  // whole multiples of 16 rows (or one sequence spans all rows); 16 / seq_rows when
  // that divides; otherwise every row may start a new sequence
  if (!row_seq || seq_rows >= M || (seq_rows > 0 && seq_rows % 16 == 0)) a.segs = 1;
  else if (seq_rows > 0 && 16 % seq_rows == 0) a.segs = 16 / seq_rows;
  else if (seq_rows > 0) a.segs = min(16, (15 + seq_rows - 1) / seq_rows + 1);
  else a.segs = min(16, M);
  a.err = device_error_word();
  a.qkv = nullptr;
  a.ldqkv = 0;
  a.q_norm = a.k_norm = nullptr;
  a.inv_freq = nullptr;
  a.eps = 0.f;
  a.k_new = a.v_new = nullptr;
  a.page_table = page_table;
  a.pt_stride = pt_stride;
  a.page_shift = 0;
  if (page_table) {
    if (page_size < ATT_KB || (page_size & (page_size - 1)) || pt_stride <= 0) {
      set_error("dfl_attention_paged: page_size must be a power of two >= %d (got %d)", ATT_KB, page_size);
      return DFL_ERR_INVALID;
    }
    while ((1 << a.page_shift) < page_size) ++a.page_shift;
  }
  if (fq) {
    a.qkv = static_cast<const __nv_bfloat16*>(fq->qkv);
    a.ldqkv = fq->ldqkv;
    a.q_norm = static_cast<const __nv_bfloat16*>(fq->q_norm);
    a.k_norm = static_cast<const __nv_bfloat16*>(fq->k_norm);
    a.inv_freq = fq->inv_freq;
    a.eps = fq->eps;
    a.k_new = static_cast<__nv_bfloat16*>(const_cast<void*>(k_cache));
    a.v_new = static_cast<__nv_bfloat16*>(const_cast<void*>(v_cache));
  }
  cudaStream_t st = as_stream(stream);
  if (attention_tc_ok(hd, G, gate != nullptr, fq != nullptr)) {
    const int s = launch_attention_tc(q, k_cache, v_cache, seq_stride, head_stride, pos, row_seq, kv_len, page_table,
                                      pt_stride, a.page_shift, M, Hq, Hkv, causal, a.scale_log2, a.n_chunks, a.segs,
                                      key_chunk, a.part_o, a.part_ml, out, ldo, n_tiles, a.err, st);
    if (s != DFL_OK) return s;
    return a.direct ? DFL_OK : launch_combine<128>(a, st);
  }
  switch (hd) {
    case 64: return deep ? launch_attn<64, 3>(a, n_tiles, st) : launch_attn<64, 2>(a, n_tiles, st);
    case 128: return deep ? launch_attn<128, 3>(a, n_tiles, st) : launch_attn<128, 2>(a, n_tiles, st);
    case 256: return launch_attn<256, 2>(a, n_tiles, st);
    default:
      set_error("dfl_attention: head_dim %d not supported (64, 128, 256)", hd);
      return DFL_ERR_UNSUPPORTED;
  }
}

extern "C" int dfl_attention(const void* q, const void* k_cache, const void* v_cache, int64_t seq_stride,
                             int64_t head_stride, const int32_t* pos, const int32_t* row_seq, const int32_t* kv_len,
                             int seq_rows, int M, int Hq, int Hkv, int hd, int causal, float scale, int max_kv,
                             int key_chunk, void* out,
                             int64_t ldo, const void* gate, int64_t ldg, int gate_head_stride, void* workspace,
                             size_t workspace_bytes, void* stream) {
  return attention_impl(q, k_cache, v_cache, seq_stride, head_stride, pos, row_seq, kv_len, seq_rows, M, Hq, Hkv, hd,
                        causal, scale, max_kv, key_chunk, out, ldo, gate, ldg, gate_head_stride, workspace,
                        workspace_bytes, stream, nullptr);
}

extern "C" int dfl_attention_qkv(const void* qkv, int64_t ldqkv, const void* q_norm, const void* k_norm,
                                 const float* inv_freq, float eps, void* k_cache, void* v_cache, int64_t seq_stride,
                                 int64_t head_stride, const int32_t* pos, const int32_t* row_seq, int seq_rows, int M,
                                 int Hq, int Hkv, float scale, int max_kv, int key_chunk, void* out, int64_t ldo,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  if (M == 0) return DFL_OK;
  if (!qkv || !q_norm || !k_norm || !inv_freq || ldqkv < (int64_t)(Hq + 2 * Hkv) * 128 || ldqkv % 8) {
    set_error("dfl_attention_qkv: bad projection rows or norm weights");
    return DFL_ERR_INVALID;
  }
  // every row of a sequence must sit in one 16-row tile (the tile's CTAs write the new keys
  // they read themselves): one sequence of at most 16 rows, or sequences of seq_rows rows
  // with seq_rows dividing 16
  const bool one_tile = row_seq ? (seq_rows > 0 && seq_rows <= 16 && 16 % seq_rows == 0) : M <= 16;
  if (!one_tile) {
    set_error("dfl_attention_qkv: needs every sequence's rows inside one 16-row tile (seq_rows=%d M=%d)",
              seq_rows, M);
    return DFL_ERR_UNSUPPORTED;
  }
  FusedQkv f{qkv, ldqkv, q_norm, k_norm, inv_freq, eps};
  return attention_impl(nullptr, k_cache, v_cache, seq_stride, head_stride, pos, row_seq, nullptr, seq_rows, M, Hq,
                        Hkv, 128, 1, scale, max_kv, key_chunk, out, ldo, nullptr, 0, 0, workspace, workspace_bytes,
                        stream, &f);
}

extern "C" int dfl_attention_paged(const void* q, const void* k_pages, const void* v_pages, int64_t page_stride,
                                   int64_t head_stride, const int32_t* page_table, int64_t pt_stride, int page_size,
                                   const int32_t* pos, const int32_t* row_seq, const int32_t* kv_len, int seq_rows,
                                   int M, int Hq, int Hkv, int hd, int causal, float scale, int max_kv, int key_chunk,
                                   void* out, int64_t ldo, const void* gate, int64_t ldg, int gate_head_stride,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  if (!page_table) {
    set_error("dfl_attention_paged: null page table");
    return DFL_ERR_INVALID;
  }
  return attention_impl(q, k_pages, v_pages, page_stride, head_stride, pos, row_seq, kv_len, seq_rows, M, Hq, Hkv, hd,
                        causal, scale, max_kv, key_chunk, out, ldo, gate, ldg, gate_head_stride, workspace,
                        workspace_bytes, stream, nullptr, page_table, pt_stride, page_size);
}

extern "C" int dfl_attention_launches(int Hq, int Hkv, int hd, int max_kv, int key_chunk) {
  if (Hkv <= 0 || Hq % Hkv || max_kv <= 0 || (hd != 64 && hd != 128 && hd != 256)) return -1;
  key_chunk = resolve_key_chunk(key_chunk);
  return (max_kv + key_chunk - 1) / key_chunk <= 1 ? 1 : 2;
}
