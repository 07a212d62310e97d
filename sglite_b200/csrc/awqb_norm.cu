// RMSNorm and residual-add RMSNorm, the step that follows a row-parallel
// projection's all-reduce.
//
// Reference behaviour (layers/norm.py:10-47): RMSNorm.forward calls
// flashinfer.rmsnorm(x, w, eps); RMSNormFused.forward(x, residual) calls
// flashinfer.fused_add_rmsnorm(x, residual, w, eps) in place. The arithmetic
// is that of flashinfer 0.6.11 (include/flashinfer/norm.cuh), restated:
//   x        = float(input) + float(residual)      (fp32)
//   residual = (T) x
//   out      = (T) (x * rsqrt(sum(x * x) / d + eps) * float(w))
// where the sum of squares is taken over the fp32 x (not the rounded residual).
// Plain RMSNorm is the same without the residual.
//
// B200 layout: one CTA per row, 512 threads, 16-byte vectors (8 fp16/bf16);
// the row stays in registers between the sum and the scaling (up to 16384
// features), so each element is read once and written once. Launched with
// programmatic dependent launch: the CTA waits for the producing kernel
// (griddepcontrol.wait) before it reads, and lets the next kernel start its
// prologue early.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "awqb200.h"
#include "awqb_common.h"

namespace awqb {
namespace {

constexpr int kNormThreads = 512;
constexpr int kNormVec = 8;                                    // elements per 16-byte vector
constexpr int kNormMaxIter = 4;                                // vectors per thread
constexpr int kNormMaxN = kNormThreads * kNormVec * kNormMaxIter;  // 16384 features

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = (float)h[j];
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int j = 0; j < 8; ++j) h[j] = (T)f[j];
  return u;
}

// Sum over the CTA (warp shuffles, then the warp totals).
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kNormThreads / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// residual == nullptr: plain RMSNorm of input into out.
// otherwise: residual += input (stored rounded), out = RMSNorm(sum) (out may be input).
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
add_rmsnorm_kernel(const T* input, T* residual, const T* __restrict__ weight, T* out, int N, int64_t ld_in,
                   int64_t ld_res, int64_t ld_out, float eps) {
  __shared__ float red[kNormThreads / 32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t row = blockIdx.x;
  const uint4* in_v = reinterpret_cast<const uint4*>(input + row * ld_in);
  uint4* res_v = residual ? reinterpret_cast<uint4*>(residual + row * ld_res) : nullptr;
  const int nvec = N / kNormVec;
  // Every load of the thread is issued before its first store (the residual
  // store could alias later loads as far as the compiler knows).
  uint4 raw_x[kNormMaxIter], raw_r[kNormMaxIter];
#pragma unroll
  for (int it = 0; it < kNormMaxIter; ++it) {
    const int vi = it * kNormThreads + threadIdx.x;
    if (vi < nvec) {
      raw_x[it] = in_v[vi];
      if (res_v != nullptr) raw_r[it] = res_v[vi];
    }
  }
  float x[kNormMaxIter][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < kNormMaxIter; ++it) {
    const int vi = it * kNormThreads + threadIdx.x;
    if (vi < nvec) {
      unpack8<T>(raw_x[it], x[it]);
      if (res_v != nullptr) {
        float r[8];
        unpack8<T>(raw_r[it], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) x[it][j] += r[j];
        res_v[vi] = pack8<T>(x[it]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += x[it][j] * x[it][j];
    }
  }
  const float total = block_sum(ss, red);
  const float rcp = rsqrtf(total / (float)N + eps);
  uint4* out_v = reinterpret_cast<uint4*>(out + row * ld_out);
  const uint4* w_v = reinterpret_cast<const uint4*>(weight);
#pragma unroll
  for (int it = 0; it < kNormMaxIter; ++it) {
    const int vi = it * kNormThreads + threadIdx.x;
    if (vi < nvec) {
      float w[8], o[8];
      unpack8<T>(w_v[vi], w);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = x[it][j] * rcp * w[j];
      out_v[vi] = pack8<T>(o);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

int norm_impl(const void* input, void* residual, const void* weight, void* out, int64_t M, int64_t N,
              int64_t ld_in, int64_t ld_res, int64_t ld_out, float eps, int dtype, void* stream) {
  AWQB_REQUIRE(M >= 0 && N > 0 && N % kNormVec == 0 && N <= kNormMaxN, kInvalidArgument,
               "N=%lld must be a positive multiple of %d, at most %d", (long long)N, kNormVec, kNormMaxN);
  AWQB_REQUIRE(ld_in >= N && ld_out >= N && (residual == nullptr || ld_res >= N) && ld_in % kNormVec == 0 &&
                   ld_out % kNormVec == 0 && ld_res % kNormVec == 0,
               kInvalidArgument, "row strides must be >= N and multiples of %d", kNormVec);
  AWQB_REQUIRE(eps >= 0.f, kInvalidArgument, "eps must be >= 0");
  if (M == 0) return kOk;
  AWQB_REQUIRE(input && weight && out, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(((uintptr_t)input & 15) == 0 && ((uintptr_t)weight & 15) == 0 && ((uintptr_t)out & 15) == 0 &&
                   ((uintptr_t)residual & 15) == 0,
               kInvalidArgument, "tensors must be 16-byte aligned");
  AWQB_REQUIRE(M <= 0x7fffffff, kInvalidArgument, "too many rows");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)M);
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dtype == AWQB_DTYPE_F16) {
    AWQB_CUDA(cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<__half>, static_cast<const __half*>(input),
                                 static_cast<__half*>(residual), static_cast<const __half*>(weight),
                                 static_cast<__half*>(out), (int)N, ld_in, ld_res, ld_out, eps));
  } else if (dtype == AWQB_DTYPE_BF16) {
    AWQB_CUDA(cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<__nv_bfloat16>,
                                 static_cast<const __nv_bfloat16*>(input), static_cast<__nv_bfloat16*>(residual),
                                 static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
                                 (int)N, ld_in, ld_res, ld_out, eps));
  } else {
    AWQB_REQUIRE(false, kInvalidArgument, "bad dtype %d", dtype);
  }
  AWQB_LAUNCH_CHECK();
  return kOk;
}

}  // namespace
}  // namespace awqb

using namespace awqb;

extern "C" int awqb_rmsnorm(const void* input, const void* weight, void* out, int64_t M, int64_t N, int64_t ld_in,
                            int64_t ld_out, float eps, int dtype, void* stream) {
  return norm_impl(input, nullptr, weight, out, M, N, ld_in, N, ld_out, eps, dtype, stream);
}

extern "C" int awqb_fused_add_rmsnorm(void* input, void* residual, const void* weight, int64_t M, int64_t N,
                                      int64_t ld_in, int64_t ld_res, float eps, int dtype, void* stream) {
  AWQB_REQUIRE(residual != nullptr || M == 0, kInvalidArgument, "residual is null");
  return norm_impl(input, residual, weight, input, M, N, ld_in, ld_res, ld_in, eps, dtype, stream);
}
