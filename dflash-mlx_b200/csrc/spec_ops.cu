// Device-side speculative-step control: greedy argmax, longest-prefix accept,
// bonus token, commit, stop detection and cache-length rollback.
//
// Reference behaviour restated here (dflash_mlx/runtime.py):
//   sample_tokens (temperature 0)          runtime.py:22-29   argmax, lowest index on ties
//   longest_prefix_match                   runtime.py:41-47
//   parallel-replay accept / bonus         runtime.py:139-163 accepted = matched + 1, bonus = posterior[matched]
//   rewind_kv_caches / trim_draft_cache    adapters.py:697-700, runtime.py:32-34, 420
//   commit + stop scan + length limit      runtime.py:488-507
// The reference pulls the posterior to the host (.tolist()) and runs these in
// Python; here they run on the device and the host only polls a status record.
// Cache rollback is a length update: the target cache length is state.start, the
// draft cache length is state.draft_len, and slots past a length are dead.
#include "common.cuh"

namespace dfl {

struct ArgmaxPair {
  float v;
  int i;
};

__device__ __forceinline__ ArgmaxPair better(ArgmaxPair a, ArgmaxPair b) {
  return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}

// argmax over the per-tile partials of one row, computed by one warp
// (the order of value desc, index asc is total, so any reduction order gives the same pair;
// eight loads per lane are kept in flight)
__device__ __forceinline__ int warp_row_argmax(const float2* part, int n_tiles, int lane) {
  ArgmaxPair best{-INFINITY, 0x7fffffff};
  int j = lane;
  for (; j + 7 * 32 < n_tiles; j += 8 * 32) {
    float2 p[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) p[u] = part[j + u * 32];
#pragma unroll
    for (int u = 0; u < 8; ++u) best = better(best, ArgmaxPair{p[u].x, __float_as_int(p[u].y)});
  }
  for (; j < n_tiles; j += 32) {
    const float2 p = part[j];
    best = better(best, ArgmaxPair{p.x, __float_as_int(p.y)});
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgmaxPair other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
    best = better(best, other);
  }
  return best.i;
}

// Argmax of rows first .. first + n - 1 of the per-tile partials by the whole block: each
// row gets nw = warps / n warps (at least one), warp `sub` of a row takes every nw-th run
// of 32 partials with sixteen loads per lane in flight, and the warps' pairs meet in shared
// memory. The (value desc, index asc) order is total, so the split does not change the
// result. Every thread of the block must call it; out[k] gets row first + k's index.
__device__ __forceinline__ void block_rows_argmax(const float2* part, int n_tiles, int first, int n, int* out) {
  __shared__ ArgmaxPair pairs[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  const int nw = max(1, warps / n);
  for (int k0 = 0; k0 < n; k0 += warps / nw) {
    const int k = k0 + warp / nw, sub = warp % nw;
    ArgmaxPair best{-INFINITY, 0x7fffffff};
    if (k < n && warp / nw < warps / nw) {
      const float2* row = part + (long long)(first + k) * n_tiles;
      const int step = 32 * nw;
      int j = sub * 32 + lane;
      for (; j + 15 * step < n_tiles; j += 16 * step) {
        float2 p[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) p[u] = row[j + u * step];
#pragma unroll
        for (int u = 0; u < 16; ++u) best = better(best, ArgmaxPair{p[u].x, __float_as_int(p[u].y)});
      }
      for (; j < n_tiles; j += step) {
        const float2 p = row[j];
        best = better(best, ArgmaxPair{p.x, __float_as_int(p.y)});
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        ArgmaxPair other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
        best = better(best, other);
      }
    }
    if (lane == 0) pairs[warp] = best;
    __syncthreads();
    if (threadIdx.x < warps / nw && k0 + (int)threadIdx.x < n) {
      ArgmaxPair b = pairs[threadIdx.x * nw];
      for (int u = 1; u < nw; ++u) b = better(b, pairs[threadIdx.x * nw + u]);
      out[k0 + threadIdx.x] = b.i;
    }
    __syncthreads();
  }
}

__global__ void argmax_reduce_kernel(const float2* __restrict__ part, int M, int n_tiles, int* __restrict__ out) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= M) return;
  const int idx = warp_row_argmax(part + (long long)row * n_tiles, n_tiles, lane);
  if (lane == 0) out[row] = idx;
}

// Per sequence: block = [out[start], mask, ...]; positions for the draft context
// rows, the draft block rows and the verify rows; draft attention length.
__global__ void step_prepare_kernel(dfl_seq_state* st, const int* __restrict__ out_tokens, long long out_stride,
                                    int* __restrict__ block, int bs, int mask_id, int* __restrict__ tpos,
                                    int* __restrict__ dpos_ctx, int* __restrict__ dpos_blk,
                                    int* __restrict__ draft_kv_len, int B) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int b = blockIdx.x;
  if (b >= B) return;
  const dfl_seq_state s = st[b];
  const bool live = !s.finished;
  for (int i = threadIdx.x; i < bs; i += blockDim.x) {
    const int r = b * bs + i;
    block[r] = i == 0 ? out_tokens[(long long)b * out_stride + s.start] : mask_id;
    tpos[r] = live ? s.start + i : -1;
    if (dpos_ctx) dpos_ctx[r] = (live && i < s.pending) ? s.draft_len + i : -1;
    if (dpos_blk) dpos_blk[r] = live ? s.draft_len + s.pending + i : -1;
  }
  if (threadIdx.x == 0 && draft_kv_len) draft_kv_len[b] = s.draft_len + s.pending + bs;
}

// Draft proposal: block[1:] = argmax of draft logits rows 1..bs-1 (runtime.py:417-423),
// optionally overridden by injected tokens; the context rows now live in the
// draft cache (draft_len += pending) and the block rows are trimmed (runtime.py:420).
__global__ void draft_commit_kernel(dfl_seq_state* st, const float2* __restrict__ part, int n_tiles,
                                    int* __restrict__ block, int bs, const int* __restrict__ inject_tokens,
                                    long long inject_stride, const int* __restrict__ inject_len,
                                    long long inject_len_stride, const int* __restrict__ inject_noise,
                                    long long noise_stride, int B) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int b = blockIdx.x;
  if (b >= B) return;
  __shared__ int post[64];
  const dfl_seq_state s = st[b];
  block_rows_argmax(part, n_tiles, b * bs + 1, bs - 1, post);  // also under injection: the same work as a real step
  __syncthreads();
  for (int i = 1 + (int)threadIdx.x; i < bs; i += blockDim.x) {
    int tok;
    if (inject_tokens) {
      const int L = inject_len[(long long)b * inject_len_stride + s.steps];
      tok = (i - 1 < L) ? inject_tokens[(long long)b * inject_stride + s.start + i]
                        : inject_noise[(long long)b * noise_stride + (long long)s.steps * bs + i];
    } else {
      tok = post[i - 1];
    }
    block[b * bs + i] = tok;
  }
  __syncthreads();
  if (threadIdx.x == 0 && !s.finished) {
    st[b].draft_len = s.draft_len + s.pending;
    st[b].pending = 0;
  }
}

// Verify accept: posterior = argmax rows; matched = LCP(block[1:], posterior[:-1]);
// accepted = matched + 1; bonus = posterior[matched]; commit; stop / length checks.
__global__ void verify_accept_kernel(dfl_seq_state* st, const float2* __restrict__ part, int n_tiles,
                                     const int* __restrict__ block, int bs, int* __restrict__ out_tokens,
                                     long long out_stride, int* __restrict__ posterior, const int* __restrict__ stop_ids,
                                     int n_stop, int* __restrict__ accept_log, long long log_stride, int B) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  __shared__ int post[64];
  const int b = blockIdx.x;
  if (b >= B) return;
  block_rows_argmax(part, n_tiles, b * bs, bs, post);
  if (posterior)
    for (int i = threadIdx.x; i < bs; i += blockDim.x) posterior[b * bs + i] = post[i];
  __syncthreads();
  if (threadIdx.x != 0) return;
  dfl_seq_state s = st[b];
  if (s.finished) {
    st[b].accepted = 0;  // recurrent-state rollback skips finished sequences
    return;
  }
  const int* blk = block + b * bs;
  int matched = 0;
  while (matched < bs - 1 && blk[matched + 1] == post[matched]) ++matched;
  const int acc = matched + 1;
  const int bonus = post[matched];
  int* out = out_tokens + (long long)b * out_stride;
  for (int i = 1; i < acc; ++i) out[s.start + i] = blk[i];
  out[s.start + acc] = bonus;
  for (int i = s.start + 1; i <= s.start + acc && s.stop_index < 0; ++i) {
    for (int j = 0; j < n_stop; ++j)
      if (out[i] == stop_ids[j]) {
        s.stop_index = i;
        break;
      }
  }
  if (accept_log) accept_log[(long long)b * log_stride + s.steps] = acc;
  s.start += acc;
  s.pending = acc;
  s.accepted = acc;
  s.bonus = bonus;
  s.steps += 1;
  if (s.stop_index >= 0 || s.start + 1 > s.total_max) s.finished = 1;
  st[b] = s;
}

// Sampling keys: row b * bs + i of a step predicts the token at absolute position
// start + i + offset of sequence b (offset 1 for verify rows, 0 for draft rows); its key
// depends on (seed, b, that position, tag) only, so a plain decode and a speculative
// decode draw the same noise for the same position.
__global__ void sample_keys_kernel(const dfl_seq_state* st, int B, int bs, unsigned long long seed, int tag, int offset,
                                   unsigned long long* keys) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * bs) return;
  const int b = r / bs, i = r % bs;
  const long long pos = (long long)st[b].start + i + offset;
  keys[r] = mix64(mix64(mix64(seed ^ (unsigned long long)tag) ^ (unsigned long long)b) ^ (unsigned long long)pos);
}

// Gumbel-max partials from logits: for row m and its 32-column group, (max over the group
// of bf16(logit) * inv_t + gumbel(key[m], column), lowest index) -- the DFL_EPI_ARGMAX
// partial layout, so argmax_reduce / draft_commit / verify_accept consume it unchanged.
__global__ void sample_partials_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, int M, int V,
                                       const unsigned long long* __restrict__ keys, float inv_t, float2* __restrict__ part) {
  grid_dependency_launch_dependents();
  grid_dependency_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (V + 31) / 32;
  const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (item >= (long long)M * groups) return;
  const int m = (int)(item / groups), grp = (int)(item % groups);
  const int n = grp * 32 + lane;
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  if (n < V) {
    best = round_bf16(__bfloat162float(logits[(long long)m * ld + n])) * inv_t + gumbel_noise(keys[m], n);
    bidx = n;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    if (ob > best || (ob == best && oi < bidx)) {
      best = ob;
      bidx = oi;
    }
  }
  if (lane == 0) part[(long long)m * groups + grp] = make_float2(best, __int_as_float(bidx));
}

static int launch_simple(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t stream, const char* what) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

}  // namespace dfl

using namespace dfl;

extern "C" int dfl_argmax_reduce(const void* partials, int M, int n_tiles, int32_t* out, void* stream) {
  if (M == 0) return DFL_OK;
  if (!partials || !out || n_tiles <= 0) {
    set_error("dfl_argmax_reduce: bad arguments");
    return DFL_ERR_INVALID;
  }
  const float2* p = static_cast<const float2*>(partials);
  void* args[] = {&p, &M, &n_tiles, &out};
  return launch_simple((const void*)argmax_reduce_kernel, dim3((M + 7) / 8), dim3(256), args, as_stream(stream),
                       "dfl_argmax_reduce");
}

extern "C" int dfl_sample_keys(const dfl_seq_state* state, int B, int bs, uint64_t seed, int tag, int offset,
                               uint64_t* keys, void* stream) {
  if (B == 0) return DFL_OK;
  if (!state || !keys || B < 0 || bs < 1) {
    set_error("dfl_sample_keys: bad arguments");
    return DFL_ERR_INVALID;
  }
  unsigned long long sd = seed;
  unsigned long long* k = reinterpret_cast<unsigned long long*>(keys);
  void* args[] = {&state, &B, &bs, &sd, &tag, &offset, &k};
  return launch_simple((const void*)sample_keys_kernel, dim3((B * bs + 127) / 128), dim3(128), args,
                       as_stream(stream), "dfl_sample_keys");
}

extern "C" int dfl_sample_partials(const void* logits, int64_t ld, int M, int V, const uint64_t* keys,
                                   float inv_temperature, void* partials, void* stream) {
  if (M == 0) return DFL_OK;
  if (!logits || !keys || !partials || M < 0 || V <= 0 || ld < V || !(inv_temperature > 0.f)) {
    set_error("dfl_sample_partials: bad arguments");
    return DFL_ERR_INVALID;
  }
  const __nv_bfloat16* lg = static_cast<const __nv_bfloat16*>(logits);
  long long l = ld;
  const unsigned long long* k = reinterpret_cast<const unsigned long long*>(keys);
  float2* p = static_cast<float2*>(partials);
  void* args[] = {&lg, &l, &M, &V, &k, &inv_temperature, &p};
  const long long items = (long long)M * ((V + 31) / 32);
  return launch_simple((const void*)sample_partials_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), args,
                       as_stream(stream), "dfl_sample_partials");
}

extern "C" int dfl_step_prepare(dfl_seq_state* state, const int32_t* out_tokens, int64_t out_stride, int32_t* block,
                                int bs, int mask_id, int32_t* target_pos, int32_t* draft_ctx_pos,
                                int32_t* draft_block_pos, int32_t* draft_kv_len, int B, void* stream) {
  if (B == 0) return DFL_OK;
  if (!state || !out_tokens || !block || !target_pos || bs < 1 || bs > 64 || B < 0) {
    set_error("dfl_step_prepare: bad arguments");
    return DFL_ERR_INVALID;
  }
  long long os = out_stride;
  void* args[] = {&state, &out_tokens, &os, &block, &bs, &mask_id, &target_pos, &draft_ctx_pos, &draft_block_pos,
                  &draft_kv_len, &B};
  return launch_simple((const void*)step_prepare_kernel, dim3(B), dim3(64), args, as_stream(stream),
                       "dfl_step_prepare");
}

extern "C" int dfl_draft_commit(dfl_seq_state* state, const void* partials, int n_tiles, int32_t* block, int bs,
                                const int32_t* inject_tokens, int64_t inject_stride, const int32_t* inject_len,
                                int64_t inject_len_stride, const int32_t* inject_noise, int64_t noise_stride, int B,
                                void* stream) {
  if (B == 0) return DFL_OK;
  if (!state || !partials || !block || bs < 1 || bs > 64 || n_tiles <= 0 ||
      (inject_tokens && (!inject_len || !inject_noise))) {
    set_error("dfl_draft_commit: bad arguments");
    return DFL_ERR_INVALID;
  }
  const float2* p = static_cast<const float2*>(partials);
  long long is = inject_stride, ils = inject_len_stride, ns = noise_stride;
  void* args[] = {&state, &p, &n_tiles, &block, &bs, &inject_tokens, &is, &inject_len, &ils, &inject_noise, &ns, &B};
  return launch_simple((const void*)draft_commit_kernel, dim3(B), dim3(1024), args, as_stream(stream),
                       "dfl_draft_commit");
}

extern "C" int dfl_verify_accept(dfl_seq_state* state, const void* partials, int n_tiles, const int32_t* block, int bs,
                                 int32_t* out_tokens, int64_t out_stride, int32_t* posterior, const int32_t* stop_ids,
                                 int n_stop, int32_t* accept_log, int64_t log_stride, int B, void* stream) {
  if (B == 0) return DFL_OK;
  if (!state || !partials || !block || !out_tokens || bs < 1 || bs > 64 || n_tiles <= 0 || n_stop < 0 ||
      (n_stop > 0 && !stop_ids)) {
    set_error("dfl_verify_accept: bad arguments");
    return DFL_ERR_INVALID;
  }
  const float2* p = static_cast<const float2*>(partials);
  long long os = out_stride, ls = log_stride;
  void* args[] = {&state, &p, &n_tiles, &block, &bs, &out_tokens, &os, &posterior, &stop_ids, &n_stop, &accept_log,
                  &ls, &B};
  return launch_simple((const void*)verify_accept_kernel, dim3(B), dim3(1024), args, as_stream(stream),
                       "dfl_verify_accept");
}
