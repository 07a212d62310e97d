// MoE routing and glue kernels around the grouped AWQ GEMM.
//
// Reference behaviour (layers/fused_moe/fused.py):
//   fused_topk (:11-31)          softmax over router logits, top-k, optional
//                                renormalisation (inside topk_softmax), then a
//                                second division by (sum + 1e-8) (:26-27).
//   moe_align_block_size (:34-61) (token, k) pairs sorted by expert, each
//                                expert's list padded to the block size with the
//                                sentinel M*topk; one expert id per block.
//   silu_and_mul (activation.py:11-15), moe_sum_reduce (triton/fused_moe.py:7-50).
// Expert parallelism (experts [e_begin, e_end) on this rank) is new here: pairs
// routed to other ranks' experts are dropped from the local sort and the sum.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "awqb200.h"
#include "awqb_common.h"

namespace awqb {
namespace {

constexpr int kMaxExperts = 512;

__device__ __forceinline__ int cmin_i(int a, int b) { return a < b ? a : b; }
constexpr int kMaxTopk = 32;

// One warp per token. Top-k is chosen on the logits (softmax is monotonic),
// ties going to the lower expert index, so the choice does not depend on the
// rounding of exp. The row lives in registers (expert e = lane + 32 j in slot
// j, taken experts in a bit mask); lane k keeps the k-th choice. Every sum runs
// in the same order as a sequential pass (experts ascending per lane, then the
// shuffle tree; choices in rank order).
__global__ void topk_softmax_kernel(const float* __restrict__ logits, int M, int E, int topk,
                                    int renormalize, float* __restrict__ w_out,
                                    int32_t* __restrict__ id_out) {
  constexpr int kSlots = kMaxExperts / 32;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= M) return;
  const float* row = logits + (int64_t)warp * E;
  float v[kSlots];
#pragma unroll
  for (int j = 0; j < kSlots; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? row[e] : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kSlots; ++j)
    if (lane + 32 * j < E) mx = fmaxf(mx, v[j]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kSlots; ++j)
    if (lane + 32 * j < E) sum += expf(v[j] - mx);
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);

  uint32_t taken = 0;
  float my_w = 0.f;
  int my_i = 0;
  float wsum = 0.f;
  for (int k = 0; k < topk; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kSlots; ++j) {
      const int e = lane + 32 * j;
      if (e >= E || (taken & (1u << j))) continue;
      if (v[j] > bv || (v[j] == bv && e < bi)) { bv = v[j]; bi = e; }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    const float p = expf(bv - mx) / sum;
    if (lane == k) { my_w = p; my_i = bi; }
    wsum += p;
  }
  if (renormalize) {
    float s2 = 0.f;
    for (int k = 0; k < topk; ++k) s2 += __shfl_sync(0xffffffffu, my_w / wsum, k);
    my_w = (my_w / wsum) / (s2 + 1e-8f);
  }
  if (lane < topk) {
    w_out[(int64_t)warp * topk + lane] = my_w;
    id_out[(int64_t)warp * topk + lane] = my_i;
  }
}

// Single CTA of 1024 threads (32 warps). Warp w owns the contiguous slice
// [w*S, (w+1)*S) of the flattened (token, k) ids and emits its pairs in index
// order, so the sort is stable and deterministic.
__global__ void __launch_bounds__(1024) align_kernel(const int32_t* __restrict__ ids, int numel, int e_begin,
                                                     int e_end, int block_m, int max_padded,
                                                     int32_t* __restrict__ sorted_ids,
                                                     int32_t* __restrict__ block_expert,
                                                     int32_t* __restrict__ num_post_pad) {
  extern __shared__ int32_t sm[];
  const int E = e_end - e_begin;
  int32_t* cnt = sm;                    // [32][E] per-warp counts, then per-warp write bases
  int32_t* off = sm + 32 * E;           // [E + 1] padded offsets
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = (numel + 31) / 32;
  const int s0 = warp * slice;
  const int s1 = min(numel, s0 + slice);

  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) cnt[i] = 0;
  for (int i = threadIdx.x; i < max_padded; i += blockDim.x) sorted_ids[i] = numel;
  __syncthreads();
  for (int i = s0 + lane; i < s1; i += 32) {
    const int e = ids[i] - e_begin;
    if (e >= 0 && e < E) atomicAdd(&cnt[warp * E + e], 1);
  }
  __syncthreads();
  // Padded size of every expert (one thread per expert), then an exclusive
  // prefix sum over experts: a shuffle scan inside each warp of 32 experts and
  // a short serial pass over the (at most 16) warp totals.
  int32_t* wsum = off + E + 1;  // [32] per-warp totals of the expert scan
  for (int e0 = 0; e0 < E; e0 += blockDim.x) {
    const int e = e0 + threadIdx.x;
    int padded = 0;
    if (e < E) {
      int tot = 0;
      for (int w = 0; w < 32; ++w) tot += cnt[w * E + e];
      padded = (tot + block_m - 1) / block_m * block_m;
    }
    int incl = padded;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (threadIdx.x == 0) {
      int run = e0 == 0 ? 0 : off[e0];
      for (int w = 0; w < 32 && e0 + w * 32 < E; ++w) {
        const int t = wsum[w];
        wsum[w] = run;
        run += t;
      }
      off[cmin_i(E, e0 + (int)blockDim.x)] = run;
    }
    __syncthreads();
    if (e < E) off[e] = wsum[warp] + incl - padded;
    __syncthreads();
  }
  if (threadIdx.x == 0) *num_post_pad = off[E];
  __syncthreads();
  // per-warp write bases: off[e] + counts of lower warps
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = off[e];
    for (int w = 0; w < 32; ++w) {
      const int c = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += c;
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    for (int b = off[e] / block_m; b < off[e + 1] / block_m; ++b) block_expert[b] = e;
  }
  __syncthreads();
  for (int base = s0; base < s1; base += 32) {
    const int i = base + lane;
    const bool live = i < s1;
    int e = live ? ids[i] - e_begin : -1;
    if (e < 0 || e >= E) e = -1;
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int rank = __popc(grp & ((1u << lane) - 1u));
      sorted_ids[cnt[warp * E + e] + rank] = i;
    }
    __syncwarp();
    if (e >= 0 && (grp & ((1u << lane) - 1u)) == 0) cnt[warp * E + e] += __popc(grp);
    __syncwarp();
  }
}

// Multi-CTA variant for large inputs (same output, same stable order): one
// CTA counts each chunk of kAlignChunk ids, one CTA turns the counts into
// padded expert offsets and per-chunk write bases, and one warp per chunk
// writes its ids in index order. A single CTA would be bound by one SM's
// shared-memory atomics and match instructions.
constexpr int kAlignChunk = 1024;

__global__ void __launch_bounds__(256) align_hist_kernel(const int32_t* __restrict__ ids, int numel, int e_begin,
                                                         int E, int32_t* __restrict__ hist) {
  extern __shared__ int32_t h[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int i0 = blockIdx.x * kAlignChunk;
  int ev[kAlignChunk / 256];
#pragma unroll
  for (int j = 0; j < kAlignChunk / 256; ++j) {
    const int i = i0 + j * 256 + threadIdx.x;
    ev[j] = i < numel ? ids[i] - e_begin : -1;
  }
#pragma unroll
  for (int j = 0; j < kAlignChunk / 256; ++j)
    if (ev[j] >= 0 && ev[j] < E) atomicAdd(&h[ev[j]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[(int64_t)blockIdx.x * E + e] = h[e];
}

// One CTA, one thread per expert (blockDim = E rounded up to a warp).
__global__ void align_scan_kernel(int32_t* __restrict__ hist, int nch, int E, int block_m, int numel,
                                  int max_padded, int32_t* __restrict__ sorted_ids,
                                  int32_t* __restrict__ block_expert, int32_t* __restrict__ num_post_pad) {
  __shared__ int32_t off[kMaxExperts + 1];
  __shared__ int32_t wsum[32];
  const int e = threadIdx.x, warp = e >> 5, lane = e & 31;
  // counts of 8 chunks in flight at a time (independent loads)
  int tot = 0;
  if (e < E) {
    for (int c0 = 0; c0 < nch; c0 += 8) {
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = c0 + j < nch ? hist[(int64_t)(c0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) tot += v[j];
    }
  }
  const int padded = e < E ? (tot + block_m - 1) / block_m * block_m : 0;
  int incl = padded;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (e == 0) {
    int run = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      const int t = wsum[w];
      wsum[w] = run;
      run += t;
    }
    off[E] = run;
    *num_post_pad = run;
  }
  __syncthreads();
  if (e < E) off[e] = wsum[warp] + incl - padded;
  __syncthreads();
  if (e < E) {
    int run = off[e];
    for (int c0 = 0; c0 < nch; c0 += 8) {  // per-chunk write bases, in chunk order
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = c0 + j < nch ? hist[(int64_t)(c0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (c0 + j < nch) hist[(int64_t)(c0 + j) * E + e] = run;
        run += v[j];
      }
    }
    for (int q = off[e] + tot; q < off[e + 1]; ++q) sorted_ids[q] = numel;  // padding of this expert
    for (int b = off[e] / block_m; b < off[e + 1] / block_m; ++b) block_expert[b] = e;
  }
  for (int q = off[E] + e; q < max_padded; q += blockDim.x) sorted_ids[q] = numel;  // unused tail
}

// One warp per chunk: its ids (loaded at once) in groups of 32, in index order.
__global__ void __launch_bounds__(32) align_scatter_kernel(const int32_t* __restrict__ ids, int numel, int e_begin,
                                                           int E, const int32_t* __restrict__ bases,
                                                           int32_t* __restrict__ sorted_ids) {
  extern __shared__ int32_t wpos[];
  const int lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) wpos[e] = bases[(int64_t)blockIdx.x * E + e];
  const int i0 = blockIdx.x * kAlignChunk;
  int ev[kAlignChunk / 32];
#pragma unroll
  for (int j = 0; j < kAlignChunk / 32; ++j) {
    const int i = i0 + 32 * j + lane;
    const int e = i < numel ? ids[i] - e_begin : -1;
    ev[j] = (e >= 0 && e < E) ? e : -1;
  }
  __syncwarp();
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kAlignChunk / 32; ++j) {
    const int e = ev[j];
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    if (e >= 0) sorted_ids[wpos[e] + __popc(grp & lt)] = i0 + 32 * j + lane;
    __syncwarp();
    if (e >= 0 && (grp & lt) == 0) wpos[e] += __popc(grp);
    __syncwarp();
  }
}

// x_sorted[r] = x[sorted_ids[r] / topk] for live rows, zero for padding rows.
__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ sorted_ids,
                                   const int32_t* __restrict__ num_post_pad, int numel, int topk,
                                   int rows_max, int vec_per_row, uint4* __restrict__ out) {
  const int rows = min(*num_post_pad, rows_max);
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < (int64_t)rows * vec_per_row;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t / vec_per_row);
    const int v = (int)(t - (int64_t)r * vec_per_row);
    const int sid = sorted_ids[r];
    uint4 val = make_uint4(0, 0, 0, 0);
    if (sid < numel) val = x[(int64_t)(sid / topk) * vec_per_row + v];
    out[t] = val;
  }
}

template <typename T>
__device__ __forceinline__ float to_f(T v) { return (float)v; }

// out[r, j] = silu(in[r, j]) * in[r, I + j], computed in fp32; eight
// elements (16 bytes) per thread and iteration (I % 8 == 0).
// silu(g) = g / (1 + e^-g) with the hardware exp2 and divide approximations
// (relative error ~1e-6, far below the fp16/bf16 rounding of the result): the
// exact expf and division would make this copy-like kernel issue-bound.
template <typename T, bool kInterleaved>
__global__ void silu_and_mul_kernel(const T* __restrict__ in, int64_t rows_max,
                                    const int32_t* __restrict__ rows_dev, int I, T* __restrict__ out) {
  int64_t rows = rows_max;
  if (rows_dev != nullptr && (int64_t)*rows_dev < rows) rows = *rows_dev;
  const int iv = I / 8;
  // 32-bit index arithmetic (a 64-bit division per 16-byte vector would cost
  // more than the memory traffic); the host checks rows_max * I / 8 < 2^31.
  const uint32_t total = (uint32_t)(rows * iv);
  for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
    const uint32_t r32 = t / (uint32_t)iv;
    const int64_t r = r32;
    const int j = (int)(t - r32 * (uint32_t)iv) * 8;
    uint4 ov;
    T* o = reinterpret_cast<T*>(&ov);
    if constexpr (kInterleaved) {  // columns 2j = gate j, 2j + 1 = up j
      const uint4 a = *reinterpret_cast<const uint4*>(in + r * 2 * I + 2 * j);
      const uint4 b = *reinterpret_cast<const uint4*>(in + r * 2 * I + 2 * j + 8);
      const T* pa = reinterpret_cast<const T*>(&a);
      const T* pb = reinterpret_cast<const T*>(&b);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const T* pr = i < 4 ? pa + 2 * i : pb + 2 * (i - 4);
        const float gf = to_f(pr[0]);
        o[i] = (T)(__fdividef(gf, 1.0f + __expf(-gf)) * to_f(pr[1]));
      }
    } else {
      const uint4 gv = *reinterpret_cast<const uint4*>(in + r * 2 * I + j);
      const uint4 uv = *reinterpret_cast<const uint4*>(in + r * 2 * I + I + j);
      const T* g = reinterpret_cast<const T*>(&gv);
      const T* u = reinterpret_cast<const T*>(&uv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float gf = to_f(g[i]);
        o[i] = (T)(__fdividef(gf, 1.0f + __expf(-gf)) * to_f(u[i]));
      }
    }
    *reinterpret_cast<uint4*>(out + r * I + j) = ov;
  }
}

// out[m, h] = sum over k of in[m, k, h] (fp32 accumulate), eight features per
// thread (H % 8 == 0). With ids given, only pairs whose expert lies in
// [e_begin, e_end) are summed.
template <typename T>
__global__ void topk_sum_kernel(const T* __restrict__ in, int M, int topk, int H,
                                const int32_t* __restrict__ ids, int e_begin, int e_end,
                                T* __restrict__ out) {
  const int hv = H / 8;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < (int64_t)M * hv;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = t / hv;
    const int h = (int)(t - m * hv) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int k = 0; k < topk; ++k) {
      if (ids != nullptr) {
        const int e = ids[m * topk + k];
        if (e < e_begin || e >= e_end) continue;
      }
      const uint4 v = *reinterpret_cast<const uint4*>(in + (m * topk + k) * H + h);
      const T* vt = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += to_f(vt[i]);
    }
    uint4 ov;
    T* o = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (T)acc[i];
    *reinterpret_cast<uint4*>(out + m * H + h) = ov;
  }
}

unsigned grid1d(int64_t items, int threads) {
  int64_t b = (items + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace
}  // namespace awqb

using namespace awqb;

extern "C" int awqb_moe_topk_softmax(const float* logits, int64_t M, int64_t E, int64_t topk,
                                     int renormalize, float* topk_weights, int32_t* topk_ids,
                                     void* stream) {
  AWQB_REQUIRE(M >= 0 && E >= 1 && E <= kMaxExperts && topk >= 1 && topk <= kMaxTopk && topk <= E,
               kInvalidArgument, "bad routing sizes M=%lld E=%lld topk=%lld", (long long)M,
               (long long)E, (long long)topk);
  if (M == 0) return kOk;
  AWQB_REQUIRE(logits && topk_weights && topk_ids, kInvalidArgument, "null pointer");
  const int threads = 256;
  const unsigned blocks = (unsigned)((M * 32 + threads - 1) / threads);
  topk_softmax_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, (int)M, (int)E, (int)topk, renormalize, topk_weights, topk_ids);
  AWQB_LAUNCH_CHECK();
  return kOk;
}

extern "C" int64_t awqb_moe_max_padded(int64_t numel, int64_t num_experts, int64_t block_m) {
  return numel + num_experts * (block_m - 1);
}

extern "C" int awqb_moe_align(const int32_t* topk_ids, int64_t numel, int64_t e_begin, int64_t e_end,
                              int64_t block_m, int32_t* sorted_ids, int64_t max_padded,
                              int32_t* block_expert, int32_t* num_post_pad, void* stream) {
  const int64_t E = e_end - e_begin;
  AWQB_REQUIRE(E >= 1 && E <= kMaxExperts && e_begin >= 0, kInvalidArgument,
               "bad expert range [%lld, %lld)", (long long)e_begin, (long long)e_end);
  AWQB_REQUIRE(block_m >= 1 && numel >= 0 && numel < (1ll << 30), kInvalidArgument, "bad sizes");
  AWQB_REQUIRE(max_padded >= numel + E * (block_m - 1), kInvalidArgument,
               "sorted_ids too small: %lld < %lld", (long long)max_padded,
               (long long)(numel + E * (block_m - 1)));
  AWQB_REQUIRE(sorted_ids && block_expert && num_post_pad && (numel == 0 || topk_ids),
               kInvalidArgument, "null pointer");
  const size_t smem = (size_t)(32 * E + E + 1 + 32) * sizeof(int32_t);
  auto kern = align_kernel;
  AWQB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<1, 1024, smem, static_cast<cudaStream_t>(stream)>>>(
      topk_ids, (int)numel, (int)e_begin, (int)e_end, (int)block_m, (int)max_padded, sorted_ids,
      block_expert, num_post_pad);
  AWQB_LAUNCH_CHECK();
  return kOk;
}

extern "C" int64_t awqb_moe_align_workspace_bytes(int64_t numel, int64_t num_experts) {
  const int64_t nch = (numel + kAlignChunk - 1) / kAlignChunk;
  return nch * num_experts * (int64_t)sizeof(int32_t);
}

extern "C" int awqb_moe_align_ex(const int32_t* topk_ids, int64_t numel, int64_t e_begin, int64_t e_end,
                                 int64_t block_m, int32_t* sorted_ids, int64_t max_padded, int32_t* block_expert,
                                 int32_t* num_post_pad, void* workspace, int64_t workspace_bytes, void* stream) {
  const int64_t E = e_end - e_begin;
  AWQB_REQUIRE(E >= 1 && E <= kMaxExperts && e_begin >= 0, kInvalidArgument,
               "bad expert range [%lld, %lld)", (long long)e_begin, (long long)e_end);
  AWQB_REQUIRE(block_m >= 1 && numel >= 0 && numel < (1ll << 30), kInvalidArgument, "bad sizes");
  AWQB_REQUIRE(max_padded >= numel + E * (block_m - 1), kInvalidArgument,
               "sorted_ids too small: %lld < %lld", (long long)max_padded,
               (long long)(numel + E * (block_m - 1)));
  AWQB_REQUIRE(sorted_ids && block_expert && num_post_pad && (numel == 0 || topk_ids), kInvalidArgument,
               "null pointer");
  const int64_t need = awqb_moe_align_workspace_bytes(numel, E);
  AWQB_REQUIRE(workspace != nullptr && workspace_bytes >= need, kInvalidArgument,
               "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)need);
  const int nch = (int)((numel + kAlignChunk - 1) / kAlignChunk);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* hist = static_cast<int32_t*>(workspace);
  if (nch > 0) {
    align_hist_kernel<<<nch, 256, E * sizeof(int32_t), st>>>(topk_ids, (int)numel, (int)e_begin, (int)E, hist);
    AWQB_LAUNCH_CHECK();
  }
  const int threads = (int)((E + 31) / 32 * 32);
  align_scan_kernel<<<1, threads, 0, st>>>(hist, nch, (int)E, (int)block_m, (int)numel, (int)max_padded,
                                           sorted_ids, block_expert, num_post_pad);
  AWQB_LAUNCH_CHECK();
  if (nch > 0) {
    align_scatter_kernel<<<nch, 32, E * sizeof(int32_t), st>>>(topk_ids, (int)numel, (int)e_begin, (int)E, hist,
                                                               sorted_ids);
    AWQB_LAUNCH_CHECK();
  }
  return kOk;
}

extern "C" int awqb_moe_gather_rows(const void* x, int64_t K, const int32_t* sorted_ids,
                                    const int32_t* num_post_pad, int64_t numel, int64_t topk,
                                    int64_t rows_max, void* out, void* stream) {
  AWQB_REQUIRE(K % 8 == 0 && K > 0, kInvalidArgument, "K=%lld must be a positive multiple of 8",
               (long long)K);
  AWQB_REQUIRE(x && sorted_ids && num_post_pad && out, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0, kInvalidArgument,
               "x and out must be 16-byte aligned");
  const int vec = (int)(K / 8);
  gather_rows_kernel<<<grid1d(rows_max * vec, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(x), sorted_ids, num_post_pad, (int)numel, (int)topk, (int)rows_max,
      vec, static_cast<uint4*>(out));
  AWQB_LAUNCH_CHECK();
  return kOk;
}

namespace {
int silu_and_mul_impl(const void* in, int64_t rows_max, const int32_t* rows_dev, int64_t I, int dtype, void* out,
                      void* stream, bool interleaved) {
  AWQB_REQUIRE(I > 0 && I % 8 == 0 && rows_max >= 0, kInvalidArgument, "I=%lld must be a positive multiple of 8",
               (long long)I);
  AWQB_REQUIRE(((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0, kInvalidArgument,
               "in and out must be 16-byte aligned");
  AWQB_REQUIRE(in && out, kInvalidArgument, "null pointer");
  if (rows_max == 0) return kOk;
  AWQB_REQUIRE(rows_max * (I / 8) < (1ll << 31), kInvalidArgument, "too many elements (rows * I / 8 >= 2^31)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned g = grid1d(rows_max * (I / 8), 256);
  if (dtype == AWQB_DTYPE_F16) {
    auto k = interleaved ? silu_and_mul_kernel<__half, true> : silu_and_mul_kernel<__half, false>;
    k<<<g, 256, 0, s>>>(static_cast<const __half*>(in), rows_max, rows_dev, (int)I, static_cast<__half*>(out));
  } else if (dtype == AWQB_DTYPE_BF16) {
    auto k = interleaved ? silu_and_mul_kernel<__nv_bfloat16, true> : silu_and_mul_kernel<__nv_bfloat16, false>;
    k<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(in), rows_max, rows_dev, (int)I,
                        static_cast<__nv_bfloat16*>(out));
  } else {
    AWQB_REQUIRE(false, kInvalidArgument, "bad dtype %d", dtype);
  }
  AWQB_LAUNCH_CHECK();
  return kOk;
}
}  // namespace

extern "C" int awqb_silu_and_mul(const void* in, int64_t rows_max, const int32_t* rows_dev, int64_t I,
                                 int dtype, void* out, void* stream) {
  return silu_and_mul_impl(in, rows_max, rows_dev, I, dtype, out, stream, false);
}

extern "C" int awqb_silu_and_mul_interleaved(const void* in, int64_t rows_max, const int32_t* rows_dev, int64_t I,
                                             int dtype, void* out, void* stream) {
  return silu_and_mul_impl(in, rows_max, rows_dev, I, dtype, out, stream, true);
}

extern "C" int awqb_moe_topk_sum(const void* in, int64_t M, int64_t topk, int64_t H,
                                 const int32_t* topk_ids, int64_t e_begin, int64_t e_end, int dtype,
                                 void* out, void* stream) {
  AWQB_REQUIRE(M >= 0 && topk >= 1 && H >= 8 && H % 8 == 0, kInvalidArgument, "bad sizes (H % 8 != 0)");
  if (M == 0) return kOk;
  AWQB_REQUIRE(in && out, kInvalidArgument, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  AWQB_REQUIRE(((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0, kInvalidArgument,
               "in and out must be 16-byte aligned");
  const unsigned g = grid1d(M * (H / 8), 256);
  if (dtype == AWQB_DTYPE_F16)
    topk_sum_kernel<__half><<<g, 256, 0, s>>>(static_cast<const __half*>(in), (int)M, (int)topk, (int)H,
                                               topk_ids, (int)e_begin, (int)e_end,
                                               static_cast<__half*>(out));
  else if (dtype == AWQB_DTYPE_BF16)
    topk_sum_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(in), (int)M,
                                                      (int)topk, (int)H, topk_ids, (int)e_begin,
                                                      (int)e_end, static_cast<__nv_bfloat16*>(out));
  else
    AWQB_REQUIRE(false, kInvalidArgument, "bad dtype %d", dtype);
  AWQB_LAUNCH_CHECK();
  return kOk;
}
