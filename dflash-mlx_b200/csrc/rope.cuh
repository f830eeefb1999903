// q/k head RMSNorm + RoPE + KV append of one (row, head): the arithmetic of
// dfl_qkv_rope_append, shared by its kernel (layer_ops.cu) and the fused epilogue of
// the QKV projection GEMM (gemm_tc.cu).
#pragma once
#include "common.cuh"

namespace dfl {

// -------------------------------------------------------------------------
// q/k head RMSNorm + RoPE + KV append.
//
// qkv row layout: [q heads (Hq x q_stride, first hd of each is q) | k heads (Hkv x hd) | v heads (Hkv x hd)].
// K/V cache layout per layer: [seq][Hkv][cap][hd] bf16; the token at position p
// lives in slot p. Paged form: [page][Hkv][page_size][hd] and a page table
// [seq][pt_stride] of page indices; position p of sequence s lives in page
// table[s][p / page_size], row p % page_size. pos[r] < 0 marks a row that is
// skipped entirely.
// q_out: [M][Hq][hd] bf16.
// -------------------------------------------------------------------------
struct QkvArgs {
  const __nv_bfloat16* qkv;
  long long ldqkv;
  int q_stride;  // elements between consecutive q heads inside a row (hd, or 2*hd with an output gate)
  const int* pos;
  const int* row_seq;  // nullable: all rows belong to sequence 0
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* inv_freq;  // [rot_dim/2]
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  long long seq_stride, head_stride;  // elements
  int M, Hq, Hkv, hd, rot_dim;
  float eps;
  int do_q;  // 0: skip q heads (context rows of the draft)
  const int* page_table;  // nullable: contiguous [seq][Hkv][cap][hd] caches
  long long pt_stride;
  int page_shift;         // log2(page_size)
  long long layer_stride; // multi-layer append: elements between consecutive layers' caches
};

// element offset of (sequence, kv head, position) in a contiguous or paged cache
__device__ __forceinline__ long long kv_offset(const int* pt, long long pt_stride, int shift, long long seq_stride,
                                               long long head_stride, int seq, int h, int p, int hd) {
  if (!pt) return seq * seq_stride + h * head_stride + (long long)p * hd;
  const long long page = pt[seq * pt_stride + (p >> shift)];
  return page * seq_stride + h * head_stride + (long long)(p & ((1 << shift) - 1)) * hd;
}

// One (row, head) of the q/k head norm + RoPE + append, by one warp; buf: hd floats of
// this warp's shared memory. Shared by qkv_rope_append_kernel and the fused epilogue of
// the QKV projection (gemm_tc.cu), so both give the same bits. layer > 0 (the stacked K/V
// projection of several layers' context rows): the row's columns of that layer, its
// k_norm weight k_norm_l and its caches (layer * layer_stride further on).
__device__ __forceinline__ void qkv_rope_row(const QkvArgs& a, int row, int head, int lane, float* buf, int layer = 0,
                                             const __nv_bfloat16* k_norm_l = nullptr) {
  const int p = a.pos[row];
  if (p < 0) return;
  const int seq = a.row_seq ? a.row_seq[row] : 0;
  const __nv_bfloat16* src;
  const __nv_bfloat16* nw = nullptr;
  __nv_bfloat16* dst;
  const long long lcache = (long long)layer * a.layer_stride;
  const __nv_bfloat16* qkv_row =
      a.qkv + (long long)row * a.ldqkv + (long long)layer * (a.Hq * a.q_stride + 2 * a.Hkv * a.hd);
  if (head < a.Hq) {
    if (!a.do_q) return;
    src = qkv_row + (long long)head * a.q_stride;
    nw = a.q_norm;
    dst = a.q_out + ((long long)row * a.Hq + head) * a.hd;
  } else if (head < a.Hq + a.Hkv) {
    const int kh = head - a.Hq;
    src = qkv_row + (long long)a.Hq * a.q_stride + (long long)kh * a.hd;
    nw = k_norm_l ? k_norm_l : a.k_norm;
    dst = a.k_cache + lcache +
          kv_offset(a.page_table, a.pt_stride, a.page_shift, a.seq_stride, a.head_stride, seq, kh, p, a.hd);
  } else {
    const int vh = head - a.Hq - a.Hkv;
    src = qkv_row + (long long)a.Hq * a.q_stride + (long long)(a.Hkv + vh) * a.hd;
    dst = a.v_cache + lcache +
          kv_offset(a.page_table, a.pt_stride, a.page_shift, a.seq_stride, a.head_stride, seq, vh, p, a.hd);
    for (int i = lane; i < a.hd; i += 32) dst[i] = src[i];
    return;
  }
  float ss = 0.f;
  for (int i = lane; i < a.hd; i += 32) {
    const float f = bf2f(src[i]);
    buf[i] = f;
    ss = sq_acc(ss, f);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)a.hd + a.eps);
  for (int i = lane; i < a.hd; i += 32) buf[i] = round_bf16(bf2f(nw[i]) * (buf[i] * inv));
  __syncwarp();
  const int half = a.rot_dim >> 1;
  for (int i = lane; i < a.hd; i += 32) {
    float o = buf[i];
    if (i < a.rot_dim) {
      const int j = i < half ? i : i - half;
      float s, c;
      sincosf(rope_angle(p, a.inv_freq[j]), &s, &c);
      o = rope_rot(buf[i], i < half ? buf[i + half] : buf[i - half], c, s, i < half);
    }
    dst[i] = f2bf(o);
  }
}

}  // namespace dfl
