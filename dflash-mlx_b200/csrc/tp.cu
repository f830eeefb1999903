// Tensor parallelism for the Qwen3.5-27B hybrid (the reference's Model.shard,
// custom_qwen35_model.py:1286-1402: row-parallel out_proj / o_proj / down_proj
// followed by an all-sum, custom_qwen35_model.py:810 and shard_linear
// "sharded-to-all").
//
// B200 design: every rank's row-parallel GEMM writes its partial [M, H] fp32 into
// its own slot of a peer-mapped buffer (CUDA IPC over NVLink / NVSwitch); one
// kernel per all-sum then
//   1. publishes "partial of call e ready" into every peer's flag array
//      (system-scope release after a system fence),
//   2. waits (bounded) until every peer has published e,
//   3. reads the N partials of its row slice straight from peer memory and writes
//      h <- bf16(h + bf16(sum over ranks in rank order)), the tap copy and the
//      per-32-column sums of squares the next RMSNorm needs.
// The reduction order is fixed (rank 0 .. N-1 per element), so every rank gets the
// same bits and a row's result does not depend on how many rows the call carries
// (the speculative step and plain decode agree bit for bit, which a library
// all-reduce whose chunking follows the message size does not promise).
// Partials stay fp32 (the single-GPU path rounds once, after the full K sum; so does
// this one, after the rank sum). Partials are double-buffered by call parity: a rank passes call e's barrier only
// after every peer finished call e - 1, so the buffer of call e - 2 is free again.
// Waits are bounded: on expiry the kernel records site 401 in the device error
// word and returns.
#include "common.cuh"
#include "tma_util.cuh"

namespace dfl {

constexpr int TP_MAX_RANKS = 8;
constexpr int TP_SITE_WAIT = 401;

struct TpArgs {
  const float* parts[TP_MAX_RANKS];  // this call's partial slot on every rank (peer pointers)
  int* flags[TP_MAX_RANKS];                  // every rank's flag array [TP_MAX_RANKS] (peer pointers)
  int* epoch;                                // local call counter (advanced by the last CTA)
  int* done;                                 // local CTA completion counter
  int* err;
  __nv_bfloat16* h;
  long long ldh;
  __nv_bfloat16* tap;
  long long ldtap;
  float* sumsq_out;  // [M][H/32]
  long long slab_stride;  // elements between a rank's K-range partial slabs
  int n_slabs;
  int rank, n_ranks, M, H;
  // nullable: also write xn = RMSNorm(h) * norm_w (the next projection's input), so that
  // projection needs no norm pass of its own
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* xn;
  long long ldxn;
  float eps;
};

constexpr int TP_NORM_MAX_H = 8192;  // row width the norm-folding form holds in shared memory

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Row m, columns c0 .. c0 + 7 (one lane): the sum over ranks (rank order, then slab order)
// of the partials, h <- bf16(h + bf16(sum)), the tap copy; returns the lane's sum of squares
// of the new h values.
__device__ __forceinline__ float reduce_span(const TpArgs& a, int m, int c0) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int j = 0; j < a.n_ranks; ++j)  // rank order, then slab order: the same sum on every rank
    for (int sl = 0; sl < a.n_slabs; ++sl) {
      const float4* pp =
          reinterpret_cast<const float4*>(a.parts[j] + sl * a.slab_stride + (long long)m * a.H + c0);
      const float4 p0 = __ldcg(pp), p1 = __ldcg(pp + 1);
      acc[0] += p0.x;
      acc[1] += p0.y;
      acc[2] += p0.z;
      acc[3] += p0.w;
      acc[4] += p1.x;
      acc[5] += p1.y;
      acc[6] += p1.z;
      acc[7] += p1.w;
    }
  __nv_bfloat16* hp = a.h + (long long)m * a.ldh + c0;
  const uint4 hv = *reinterpret_cast<const uint4*>(hp);
  const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&hv);
  uint32_t pk[4];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const float y0 = bf2f(hb[i]) + round_bf16(acc[i]);
    const float y1 = bf2f(hb[i + 1]) + round_bf16(acc[i + 1]);
    pk[i / 2] = pack_bf16x2(y0, y1);
    const float q0 = round_bf16(y0), q1 = round_bf16(y1);
    ss += q0 * q0 + q1 * q1;
  }
  const uint4 out = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  *reinterpret_cast<uint4*>(hp) = out;
  if (a.tap) *reinterpret_cast<uint4*>(a.tap + (long long)m * a.ldtap + c0) = out;
  return ss;
}

// one warp per (row, 256-column span): lane owns 8 consecutive columns
template <bool NORM>
__global__ void __launch_bounds__(256) tp_reduce_residual_kernel(TpArgs a) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  __shared__ int s_ok;
  const int e = *a.epoch + 1;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();  // this rank's partial (written by the previous kernel) before the flag
      for (int j = 0; j < a.n_ranks; ++j) st_release_sys(a.flags[j] + a.rank, e);
    }
    // wait until every rank published call e
    bool ok = true;
    const long long t0 = clock64();
    for (int j = 0; j < a.n_ranks && ok; ++j) {
      while (ld_acquire_sys(a.flags[a.rank] + j) < e) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) {
          atomicCAS(a.err, 0, TP_SITE_WAIT);
          ok = false;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!NORM && s_ok) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int spans = a.H / 256;
    const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
    for (long long it = item; it < (long long)a.M * spans; it += (long long)gridDim.x * (blockDim.x >> 5)) {
      const int m = (int)(it / spans), c0 = (int)(it % spans) * 256 + lane * 8;
      float ss = reduce_span(a, m, c0);
      if (a.sumsq_out) {  // four lanes cover one 32-column group
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        if ((lane & 3) == 0) a.sumsq_out[(long long)m * (a.H / 32) + c0 / 32] = ss;
      }
    }
  }
  if (NORM && s_ok) {
    // one row at a time per CTA: the row's spans, its 32-column sums of squares into shared
    // memory, their sum in column order (the norm prologue's order), then xn
    __shared__ float s_part[TP_NORM_MAX_H / 32];
    __shared__ float s_inv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int spans = a.H / 256, n_parts = a.H / 32;
    for (int m = blockIdx.x; m < a.M; m += gridDim.x) {
      for (int sp = warp; sp < spans; sp += warps) {
        const int c0 = sp * 256 + lane * 8;
        float ss = reduce_span(a, m, c0);
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        if ((lane & 3) == 0) {
          s_part[c0 / 32] = ss;
          if (a.sumsq_out) a.sumsq_out[(long long)m * n_parts + c0 / 32] = ss;
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        float ss = 0.f;
        for (int p = 0; p < n_parts; ++p) ss += s_part[p];
        s_inv = rsqrtf(ss / (float)a.H + a.eps);
      }
      __syncthreads();
      const float inv = s_inv;
      for (int k = threadIdx.x * 8; k < a.H; k += blockDim.x * 8) {
        uint4 xv = *reinterpret_cast<const uint4*>(a.h + (long long)m * a.ldh + k);
        const uint4 wv = *reinterpret_cast<const uint4*>(a.norm_w + k);
        __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) xe[e] = f2bf(bf2f(we[e]) * (bf2f(xe[e]) * inv));
        *reinterpret_cast<uint4*>(a.xn + (long long)m * a.ldxn + k) = xv;
      }
      __syncthreads();
    }
  }
  // the last CTA advances the call counter for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(a.done, 1);
    if (prev == (int)gridDim.x - 1) {
      *a.done = 0;
      *a.epoch = e;
    }
  }
}

}  // namespace dfl

using namespace dfl;

extern "C" int dfl_tp_alloc(size_t bytes, void** ptr, unsigned char* ipc_handle_out) {
  if (!ptr || !ipc_handle_out || bytes == 0) {
    set_error("dfl_tp_alloc: bad arguments");
    return DFL_ERR_INVALID;
  }
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *ptr);
  if (e == cudaSuccess) memcpy(ipc_handle_out, &h, sizeof(h));
  if (e != cudaSuccess) {
    set_error("dfl_tp_alloc: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_tp_open(const unsigned char* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) {
    set_error("dfl_tp_open: bad arguments");
    return DFL_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("dfl_tp_open: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_tp_close(void* peer_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  if (e != cudaSuccess) {
    set_error("dfl_tp_close: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_tp_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("dfl_tp_free: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

static int tp_reduce_impl(const void* const* parts, int* const* flags, int* epoch, int* done, int rank, int n_ranks,
                          int n_slabs, int64_t slab_stride, void* h, int64_t ldh, void* tap, int64_t ldtap,
                          float* sumsq_out, int M, int H, const void* norm_w, float eps, void* xn, int64_t ldxn,
                          void* stream) {
  if (M == 0) return DFL_OK;
  if (!parts || !flags || !epoch || !done || !h || n_ranks < 1 || n_ranks > TP_MAX_RANKS || rank < 0 ||
      rank >= n_ranks || M < 0 || H <= 0 || n_slabs < 1 || (n_slabs > 1 && slab_stride < (long long)M * H) ||
      slab_stride % 4) {
    set_error("dfl_tp_reduce_residual: bad arguments");
    return DFL_ERR_INVALID;
  }
  if (H % 256 || ldh % 8 || (tap && ldtap % 8)) {
    set_error("dfl_tp_reduce_residual: H must be a multiple of 256 and rows 16-byte aligned (H=%d)", H);
    return DFL_ERR_UNSUPPORTED;
  }
  TpArgs a;
  for (int j = 0; j < TP_MAX_RANKS; ++j) {
    a.parts[j] = j < n_ranks ? static_cast<const float*>(parts[j]) : nullptr;
    a.flags[j] = j < n_ranks ? flags[j] : nullptr;
  }
  a.epoch = epoch;
  a.done = done;
  a.err = device_error_word();
  a.h = static_cast<__nv_bfloat16*>(h);
  a.ldh = ldh;
  a.tap = static_cast<__nv_bfloat16*>(tap);
  a.ldtap = ldtap;
  a.sumsq_out = sumsq_out;
  a.n_slabs = n_slabs;
  a.slab_stride = slab_stride;
  a.rank = rank;
  a.n_ranks = n_ranks;
  a.M = M;
  a.H = H;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.xn = static_cast<__nv_bfloat16*>(xn);
  a.ldxn = ldxn;
  a.eps = eps;
  const long long items = norm_w ? (long long)M * 8 : (long long)M * (H / 256);  // norm form: a row per CTA
  int blocks = (int)((items + 7) / 8);
  if (blocks > 148) blocks = 148;  // every CTA waits on the flags: keep the grid resident
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = norm_w ? cudaLaunchKernelEx(&cfg, tp_reduce_residual_kernel<true>, a)
                         : cudaLaunchKernelEx(&cfg, tp_reduce_residual_kernel<false>, a);
  if (e != cudaSuccess) {
    set_error("dfl_tp_reduce_residual: launch failed: %s", cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

extern "C" int dfl_tp_reduce_residual(const void* const* parts, int* const* flags, int* epoch, int* done, int rank,
                                      int n_ranks, int n_slabs, int64_t slab_stride, void* h, int64_t ldh, void* tap,
                                      int64_t ldtap, float* sumsq_out, int M, int H, void* stream) {
  return tp_reduce_impl(parts, flags, epoch, done, rank, n_ranks, n_slabs, slab_stride, h, ldh, tap, ldtap, sumsq_out,
                        M, H, nullptr, 0.f, nullptr, 0, stream);
}

extern "C" int dfl_tp_reduce_residual_norm(const void* const* parts, int* const* flags, int* epoch, int* done,
                                           int rank, int n_ranks, int n_slabs, int64_t slab_stride, void* h,
                                           int64_t ldh, void* tap, int64_t ldtap, float* sumsq_out, int M, int H,
                                           const void* norm_w, float eps, void* xn, int64_t ldxn, void* stream) {
  if (M > 0 && (!norm_w || !xn || H > TP_NORM_MAX_H || ldxn % 8 || ldxn < H)) {
    set_error("dfl_tp_reduce_residual_norm: needs norm_w, xn (row stride >= H, multiple of 8) and H <= %d",
              TP_NORM_MAX_H);
    return DFL_ERR_INVALID;
  }
  return tp_reduce_impl(parts, flags, epoch, done, rank, n_ranks, n_slabs, slab_stride, h, ldh, tap, ldtap, sumsq_out,
                        M, H, norm_w, eps, xn, ldxn, stream);
}
