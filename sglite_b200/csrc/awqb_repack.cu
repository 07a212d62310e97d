// Post-load repack of AWQ tensors into the blob layout (awqb_layout.cuh), its
// exact inverse, and a stand-alone dequantiser that uses the same int4 ->
// fp16/bf16 routine as the GEMM. The repack replaces the reference's
// awq_marlin_repack + marlin_permute_scales + awq_to_marlin_zero_points
// (layers/quantization/awq_marlin.py:300-319); the dequantiser restates the
// reference's unpack-and-dequantise (awq_triton.py:53-62, 94-96, 119-122).
#include <cuda_runtime.h>

#include "awqb200.h"
#include "awqb_common.h"
#include "awqb_layout.cuh"

namespace awqb {
namespace {

// AWQ stores logical column i of a packed word at bits 4 * kAwqPos[i]
// (reverse of the packing order [0, 2, 4, 6, 1, 3, 5, 7]).
__device__ __constant__ int kAwqPos[8] = {0, 4, 1, 5, 2, 6, 3, 7};

// Bit offset of k-index i (0..7) inside a blob word.
__host__ __device__ __forceinline__ int blob_shift(int i) { return (i & 1) ? 16 + 4 * (i >> 1) : 4 * (i >> 1); }

struct Geo {
  int64_t K, N, G;
  int NT, KB, gpb;
  int64_t block_bytes, blob_bytes;
};

int64_t rup(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

int make_geo(int64_t K, int64_t N, int64_t G, Geo* g) {
  AWQB_REQUIRE(K > 0 && N > 0, kInvalidArgument, "bad sizes K=%lld N=%lld", (long long)K, (long long)N);
  AWQB_REQUIRE(G == 32 || G == 64 || (G >= 128 && G % 128 == 0), kUnsupported,
               "group size %lld not supported (32, 64 or a multiple of 128)", (long long)G);
  AWQB_REQUIRE(K % G == 0, kInvalidArgument, "K=%lld not a multiple of group size %lld", (long long)K,
               (long long)G);
  AWQB_REQUIRE(N % 8 == 0, kInvalidArgument, "N=%lld not a multiple of 8", (long long)N);
  g->K = K;
  g->N = N;
  g->G = G;
  g->NT = (int)(rup(N, kBlockN) / kBlockN);
  g->KB = (int)blob_kblocks(K);
  g->gpb = groups_per_block((int)G);
  g->block_bytes = block_bytes_for_gpb(g->gpb);
  g->blob_bytes = (int64_t)g->NT * g->KB * g->block_bytes;
  return kOk;
}

// Group index held by slot g of block kb, or -1 if none.
__device__ __forceinline__ int64_t block_group(int kb, int g, int gpb, int64_t G, int64_t ngroups) {
  const int64_t gi = (G < kBlockK) ? (int64_t)kb * gpb + g : ((int64_t)kb * kBlockK) / G;
  return gi < ngroups ? gi : -1;
}

// One thread per blob word (row r, word j) of block (nt, kb).
__global__ void repack_words_kernel(const int32_t* __restrict__ qweight, uint8_t* __restrict__ blob,
                                    Geo geo) {
  const int64_t words = (int64_t)geo.NT * geo.KB * 2048;
  const int64_t b = blockIdx.y;
  const int32_t* qw = qweight + b * geo.K * (geo.N / 8);
  uint8_t* out = blob + b * geo.blob_bytes;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < words;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t & 127);
    const int j = (int)((t >> 7) & 15);
    const int64_t blk = t >> 11;  // nt * KB + kb
    const int nt = (int)(blk / geo.KB);
    const int kb = (int)(blk - (int64_t)nt * geo.KB);
    const int64_t n = (int64_t)nt * kBlockN + r;
    const int64_t k0 = (int64_t)kb * kBlockK + j * 8;
    uint32_t w = 0;
    if (n < geo.N) {
      const int sh = 4 * kAwqPos[n & 7];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t k = k0 + i;
        if (k < geo.K) {
          const uint32_t src = (uint32_t)__ldg(&qw[k * (geo.N / 8) + (n >> 3)]);
          w |= ((src >> sh) & 0xFu) << blob_shift(i);
        }
      }
    }
    reinterpret_cast<uint32_t*>(out + blk * geo.block_bytes)[word_index(r, j)] = w;
  }
}

// One thread per (block, group slot, 8-row group): eight scales + one zeros word.
__global__ void repack_sz_kernel(const int32_t* __restrict__ qzeros, const uint16_t* __restrict__ scales,
                                 uint8_t* __restrict__ blob, Geo geo) {
  const int64_t items = (int64_t)geo.NT * geo.KB * geo.gpb * 16;
  const int64_t b = blockIdx.y;
  const int64_t ngroups = geo.K / geo.G;
  const int32_t* qz = qzeros + b * ngroups * (geo.N / 8);
  const uint16_t* sc = scales + b * ngroups * geo.N;
  uint8_t* out = blob + b * geo.blob_bytes;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < items;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int r8 = (int)(t & 15);
    const int64_t rest = t >> 4;
    const int g = (int)(rest % geo.gpb);
    const int64_t blk = rest / geo.gpb;
    const int nt = (int)(blk / geo.KB);
    const int kb = (int)(blk - (int64_t)nt * geo.KB);
    const int64_t gi = block_group(kb, g, geo.gpb, geo.G, ngroups);
    uint8_t* bp = out + blk * geo.block_bytes;
    uint32_t zw = 0;
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int r = r8 * 8 + rr;
      const int64_t n = (int64_t)nt * kBlockN + r;
      uint16_t s = 0;
      uint32_t z = 0;
      if (gi >= 0 && n < geo.N) {
        s = __ldg(&sc[gi * geo.N + n]);
        const uint32_t src = (uint32_t)__ldg(&qz[gi * (geo.N / 8) + (n >> 3)]);
        z = (src >> (4 * kAwqPos[n & 7])) & 0xFu;
      }
      reinterpret_cast<uint16_t*>(bp + scale_off())[g * 128 + r] = s;
      zw |= z << (4 * rr);
    }
    reinterpret_cast<uint32_t*>(bp + zero_off(geo.gpb))[g * 16 + r8] = zw;
  }
}

__device__ __forceinline__ const uint8_t* blob_block(const uint8_t* blob, const Geo& geo, int64_t n,
                                                     int64_t k) {
  const int nt = (int)(n / kBlockN);
  const int kb = (int)(k / kBlockK);
  return blob + ((int64_t)nt * geo.KB + kb) * geo.block_bytes;
}

// Inverse of repack_words: one thread per AWQ qweight word (k, c).
__global__ void unrepack_words_kernel(const uint8_t* __restrict__ blob, int32_t* __restrict__ qweight,
                                      Geo geo) {
  const int64_t cols = geo.N / 8;
  const int64_t total = geo.K * cols;
  const int64_t b = blockIdx.y;
  const uint8_t* in = blob + b * geo.blob_bytes;
  int32_t* qw = qweight + b * total;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = t / cols;
    const int64_t c = t - k * cols;
    const int j = (int)((k % kBlockK) >> 3);
    const int ii = (int)(k & 7);
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = c * 8 + i;
      const uint8_t* bp = blob_block(in, geo, n, k);
      const uint32_t src = reinterpret_cast<const uint32_t*>(bp)[word_index((int)(n % kBlockN), j)];
      w |= ((src >> blob_shift(ii)) & 0xFu) << (4 * kAwqPos[i]);
    }
    qw[t] = (int32_t)w;
  }
}

// Inverse of repack_sz: one thread per qzeros word (group gi, column word c).
__global__ void unrepack_sz_kernel(const uint8_t* __restrict__ blob, int32_t* __restrict__ qzeros,
                                   uint16_t* __restrict__ scales, Geo geo) {
  const int64_t cols = geo.N / 8;
  const int64_t ngroups = geo.K / geo.G;
  const int64_t total = ngroups * cols;
  const int64_t b = blockIdx.y;
  const uint8_t* in = blob + b * geo.blob_bytes;
  int32_t* qz = qzeros + b * total;
  uint16_t* sc = scales + b * ngroups * geo.N;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gi = t / cols;
    const int64_t c = t - gi * cols;
    const int64_t k = gi * geo.G;  // first k of the group
    const int g = (geo.G < kBlockK) ? (int)(gi % geo.gpb) : 0;
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = c * 8 + i;
      const int r = (int)(n % kBlockN);
      const uint8_t* bp = blob_block(in, geo, n, k);
      uint16_t s;
      uint32_t z;
      block_scale_zero(bp, geo.gpb, g, r, s, z);
      sc[gi * geo.N + n] = s;
      w |= z << (4 * kAwqPos[i]);
    }
    qz[t] = (int32_t)w;
  }
}

// Dequantise the blob back to W[K, N] (row-major, activation dtype) with the
// GEMM's own routine: one thread per blob word, eight k values of one feature.
template <typename T>
__global__ void dequant_kernel(const uint8_t* __restrict__ blob, T* __restrict__ w_out, Geo geo) {
  using DQ = DqTraits<T>;
  const int64_t words = (int64_t)geo.NT * geo.KB * 2048;
  const int64_t b = blockIdx.y;
  const uint8_t* in = blob + b * geo.blob_bytes;
  T* W = w_out + b * geo.K * geo.N;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < words;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t & 127);
    const int j = (int)((t >> 7) & 15);
    const int64_t blk = t >> 11;
    const int nt = (int)(blk / geo.KB);
    const int kb = (int)(blk - (int64_t)nt * geo.KB);
    const int64_t n = (int64_t)nt * kBlockN + r;
    const int64_t k0 = (int64_t)kb * kBlockK + j * 8;
    if (n >= geo.N) continue;
    const uint8_t* bp = in + blk * geo.block_bytes;
    const int g = (j * 8 * geo.gpb) / kBlockK;
    uint16_t s;
    uint32_t z;
    block_scale_zero(bp, geo.gpb, g, r, s, z);
    const typename DQ::Terms terms = DQ::make(s, z);
    const uint32_t wd = reinterpret_cast<const uint32_t*>(bp)[word_index(r, j)];
    const uint4 o = DQ::dq8(wd, terms);
    const uint16_t* h = reinterpret_cast<const uint16_t*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t k = k0 + i;
      if (k < geo.K) reinterpret_cast<uint16_t*>(W)[k * geo.N + n] = h[i];
    }
  }
}

dim3 grid_for(int64_t items, int64_t batch) {
  int64_t blocks = (items + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  if (blocks < 1) blocks = 1;
  return dim3((unsigned)blocks, (unsigned)batch);
}

}  // namespace
}  // namespace awqb

using namespace awqb;

extern "C" int awqb_blob_bytes(int64_t K, int64_t N, int64_t G, int64_t* bytes) {
  Geo geo;
  int st = make_geo(K, N, G, &geo);
  if (st != kOk) return st;
  AWQB_REQUIRE(bytes != nullptr, kInvalidArgument, "bytes is null");
  *bytes = geo.blob_bytes;
  return kOk;
}

extern "C" int awqb_repack(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                           int64_t batch, int64_t K, int64_t N, int64_t G, void* blob, void* stream) {
  Geo geo;
  int st = make_geo(K, N, G, &geo);
  if (st != kOk) return st;
  AWQB_REQUIRE(batch >= 1 && batch <= 65535, kInvalidArgument, "batch %lld out of range", (long long)batch);
  AWQB_REQUIRE(qweight && qzeros && scales && blob, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(((uintptr_t)blob & 15) == 0, kInvalidArgument, "blob must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  repack_words_kernel<<<grid_for((int64_t)geo.NT * geo.KB * 2048, batch), 256, 0, s>>>(
      qweight, static_cast<uint8_t*>(blob), geo);
  AWQB_LAUNCH_CHECK();
  repack_sz_kernel<<<grid_for((int64_t)geo.NT * geo.KB * geo.gpb * 16, batch), 256, 0, s>>>(
      qzeros, scales, static_cast<uint8_t*>(blob), geo);
  AWQB_LAUNCH_CHECK();
  return kOk;
}

extern "C" int awqb_unrepack(const void* blob, int64_t batch, int64_t K, int64_t N, int64_t G,
                             int32_t* qweight, int32_t* qzeros, uint16_t* scales, void* stream) {
  Geo geo;
  int st = make_geo(K, N, G, &geo);
  if (st != kOk) return st;
  AWQB_REQUIRE(batch >= 1 && batch <= 65535, kInvalidArgument, "batch %lld out of range", (long long)batch);
  AWQB_REQUIRE(qweight && qzeros && scales && blob, kInvalidArgument, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unrepack_words_kernel<<<grid_for(K * (N / 8), batch), 256, 0, s>>>(
      static_cast<const uint8_t*>(blob), qweight, geo);
  AWQB_LAUNCH_CHECK();
  unrepack_sz_kernel<<<grid_for((K / G) * (N / 8), batch), 256, 0, s>>>(
      static_cast<const uint8_t*>(blob), qzeros, scales, geo);
  AWQB_LAUNCH_CHECK();
  return kOk;
}

extern "C" int awqb_dequant(const void* blob, int64_t batch, int64_t K, int64_t N, int64_t G, int dtype,
                            void* w, void* stream) {
  Geo geo;
  int st = make_geo(K, N, G, &geo);
  if (st != kOk) return st;
  AWQB_REQUIRE(batch >= 1 && batch <= 65535, kInvalidArgument, "batch %lld out of range", (long long)batch);
  AWQB_REQUIRE(blob && w, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(dtype == AWQB_DTYPE_F16 || dtype == AWQB_DTYPE_BF16, kInvalidArgument, "bad dtype %d", dtype);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid = grid_for((int64_t)geo.NT * geo.KB * 2048, batch);
  if (dtype == AWQB_DTYPE_F16)
    dequant_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(blob), static_cast<__half*>(w), geo);
  else
    dequant_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(blob),
                                                       static_cast<__nv_bfloat16*>(w), geo);
  AWQB_LAUNCH_CHECK();
  return kOk;
}
