// Small-batch (decode) W4A16 GEMM for sm_100a: y[M, N] = x[M, K] * dequant(blob)
// for M <= 32, streaming the weights at HBM speed.
//
// Replaces, for decode batches, the reference's awq_gemm_kernel with its
// SPLIT_K = 8 buffer and the .sum(0) pass (layers/quantization/awq_triton.py:
// 16-136, 173-193) and gptq_marlin_gemm (marlin_utils.py:388-410).
//
// Why a second kernel next to the tcgen05 GEMM: at small M a 128-feature x
// 16-token tcgen05.mma multiplies mostly padding, its A operand has to pass
// through tensor memory (4 bytes of tcgen05.st per int4 weight), and the few
// 128-feature tiles force a cross-CTA split-K reduction. Here each CTA owns a
// narrow slice of F output features over the whole K, so no reduction crosses
// CTAs; the weights are dequantised in registers and multiplied with
// mma.sync.m16n8k16 (the weights as operand A, 8 tokens as operand B, fp32
// accumulation), which needs no shared-memory or tensor-memory copy of the
// dequantised tile.
//
// Work of one CTA: features [F*c, F*c + F) of the output, all of K, in stages
// of W k-blocks (W = 8 or 16 compute warps; 1024 or 2048 k). One producer warp streams each stage with four
// TMA loads (packed nibbles, scales, zero points and the activations) into a
// ring of shared-memory stages; the weight loads of the first ring's worth of
// stages are issued before the programmatic-dependent-launch wait, so they
// overlap the previous kernel. Compute warp w takes k-block w of every stage;
// the W partial sums are added in the epilogue. Sixteen warps per CTA suit
// narrow outputs (few CTAs: more warps per SM), eight suit wide ones (more,
// smaller CTAs per SM).
//
// Arithmetic: the dequantiser only turns a nibble pair into the exact 16-bit
// values OFF + q (OFF = 128 for bf16, 1024 for fp16: one lop3 per pair); the
// tensor core accumulates D = sum_k (OFF + q_k) x_k over a group in fp32 (the
// first MMA of a group starts from zero) and, with an all-ones operand A,
// X = sum_k x_k; the group then adds s * (D - (OFF + z) X) to the fp32
// accumulator. This is the reference's sum of x * (q - z) * s without its
// rounding of each dequantised weight to 16 bits (the GEMM contract is
// max |y - ref| <= 1e-2 max |ref| against an fp32 accumulation of the
// reference's weights; the dequantised weights themselves stay bit-exact in
// awqb_dequant). The cancellation in D - (OFF + z) X costs at most 11 of fp32's
// 24 bits. Measured on B200: the kernel is bound by instruction issue (the
// shift + lop3 pairs run on the 64-lane integer pipe), so the loop keeps
// per-block overheads (ring bookkeeping, zero and scale unpacking, accumulator
// set-up) to a few instructions per word, takes the zero point out of the
// per-weight work (one all-ones MMA per two weight MMAs instead of four
// subtractions per word), and runs sixteen warps per CTA for narrow outputs
// (folding the scale into operand A, or more accumulator chains per group,
// measured slower). With 16 or 32 tokens the all-ones MMAs would grow with the
// token groups while the tensor pipe is already the busier one, so there the
// dequantiser subtracts OFF + z (exact: q - z as a 16-bit value) and the group
// adds s * D; this also frees the X registers (measured on B200: 5-25 % faster
// at M = 16 than the all-ones form, and no spills at M = 32).
//
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "awqb_layout.cuh"
#include "awqb_ptx.cuh"

namespace awqb {

enum GemvError : uint32_t {
  kErrGemvFull = 32u,   // a compute warp gave up waiting for a stage
  kErrGemvEmpty = 64u,  // the producer gave up waiting for a free slot
};

struct GemvParams {
  const void* bias;   // [N] activation dtype or null
  void* y;            // [M][ldy]
  int64_t ldy;
  int32_t M, N, K;
  int32_t kb_real;    // k-blocks holding real input features: ceil(K / 128)
  int32_t stages;     // ceil(kb_real / W)
  int32_t ring;       // shared-memory stages in the ring (1..16)
  int32_t silu_mul;   // interleaved gate/up columns: y[., j] = silu(col 2j) * col 2j+1
  uint32_t* err;
  // Fused all-reduce across tensor-parallel ranks (tp_world >= 1), the
  // protocol of the tcgen05 kernel's exchange (awqb_gemm.cuh, GemmParams):
  // {fp32, call tag} words into every rank's landing buffer (all-to-all) or
  // into the slice owner's only, whose rounded sums come back as {16-bit
  // value, 15-bit tag} words (reduce-scatter + all-gather; owner of CTA c's
  // slice = rank c % world). Sums are taken in rank order on every rank.
  int32_t tp_world, tp_rank, tp_rows, tp_rsag;
  int64_t tp_half, tp_fhalf;    // landing / final words per parity half
  uint2* tp_land[8];
  uint32_t* tp_final[8];
  int32_t* tp_epoch;            // call counter (tag = epoch + 1, buffer = epoch & 1) and CTAs done
};

template <int F, int MT, int GPB, int W>
struct GemvCfg {
  static constexpr int kWarps = W;                      // compute warps, one k-block each per stage
  static constexpr int kThreads = 32 * (kWarps + 1);    // + the producer warp
  static constexpr int kSB = W;                         // k-blocks per stage
  static constexpr int kRG = F / 16;                    // MMA row groups (16 features)
  static constexpr int kTG = MT / 8;                    // token groups of the MMA's N = 8
  static constexpr int kZWords = F / 8 < 4 ? 4 : F / 8; // zero-point words fetched per (block, group)
  static constexpr int kWBytes = kSB * 4 * F * 16;      // packed nibbles: [block][quarter][F][16 B]
  static constexpr int kSBytes = kSB * GPB * F * 2;     // scales: [block][group][F] u16
  static constexpr int kZBytes = kSB * GPB * kZWords * 4;
  __host__ __device__ static constexpr int r128(int b) { return (b + 127) / 128 * 128; }
  static constexpr int kSOff = r128(kWBytes);
  static constexpr int kZOff = kSOff + r128(kSBytes);
  static constexpr int kXOff = kZOff + r128(kZBytes);
  static constexpr uint32_t kWeightTx = kWBytes + kSBytes + kZBytes;
  // Activations per stage: [4 W chunks of 32 k][M rows][64 B].
  __host__ __device__ static constexpr int x_bytes(int M) { return kSB * 4 * M * 64; }
  __host__ __device__ static constexpr int stage_bytes(int M) { return kXOff + r128(x_bytes(M)); }
  static constexpr int kRedBytes = kWarps * F * MT * 4;  // cross-warp reduction (reuses the ring)
  static_assert(F % 16 == 0 && F >= 16 && F <= 64, "feature slice is 16, 32 or 64");
  static_assert(MT == 8 || MT == 16 || MT == 32, "8, 16 or 32 tokens");
  static_assert(GPB == 1 || GPB == 2 || GPB == 4, "groups per block");
  static_assert(W == 8 || W == 16, "8 or 16 compute warps");
};

template <typename T> struct GemvTraits;
template <> struct GemvTraits<__half> {
  static constexpr uint32_t kMagic = 0x64006400u;  // 1024 in both halves: OR-ing q gives 1024 + q
  static constexpr uint32_t kOnes = 0x3C003C00u;   // 1.0 in both halves
  static constexpr float kOff = 1024.0f;
  // (1024 + z) in both halves, exact
  __device__ __forceinline__ static uint32_t zero2(uint32_t z) { return (0x6400u | z) * 0x00010001u; }
  __device__ __forceinline__ static uint32_t sub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  __device__ __forceinline__ static float to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  __device__ __forceinline__ static uint16_t from_f32(float v) { return __half_as_ushort(__float2half_rn(v)); }
};
template <> struct GemvTraits<__nv_bfloat16> {
  static constexpr uint32_t kMagic = 0x43004300u;  // 128 in both halves: OR-ing q gives 128 + q
  static constexpr uint32_t kOnes = 0x3F803F80u;   // 1.0 in both halves
  static constexpr float kOff = 128.0f;
  __device__ __forceinline__ static uint32_t zero2(uint32_t z) { return (0x4300u | z) * 0x00010001u; }
  __device__ __forceinline__ static uint32_t sub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  __device__ __forceinline__ static float to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
  __device__ __forceinline__ static uint16_t from_f32(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
};

// D += A * B, m16n8k16, fp32 accumulators, 16-bit inputs of type T.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B (accumulator input zero).
template <typename T>
__device__ __forceinline__ void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816_z<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}
template <>
__device__ __forceinline__ void mma16816_z<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                   uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.b16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// Nibble pair p of a blob word as two exact 16-bit values OFF + q.
template <uint32_t MAGIC>
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int p) {
  uint32_t r;
  const uint32_t s = w >> (4 * p);
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(s), "r"(0x000F000Fu), "r"(MAGIC));
  return r;
}

// 4-D tiled TMA load (no multicast); c0 is the innermost coordinate.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(policy)
      : "memory");
}

// Fused all-reduce epilogue of one CTA's slice (compute warps only; red holds
// the W per-warp partial sums [warp][token][F]). Two passes: every partial
// goes out first, then each thread waits (bounded) for the words of the values
// it sent, sums them in rank order, adds the bias once and stores; in
// reduce-scatter mode non-owners wait for the owner's rounded result instead.
// The last CTA to finish advances the rank's call counter.
template <typename T, int F, int MT>
__device__ __noinline__ void gemv_exchange(const GemvParams& p, const float* red, int f0, int nwarps) {
  using Tr = GemvTraits<T>;
  const int nthreads = 32 * nwarps;
  const int tid = threadIdx.x;
  const int M = p.M;
  grid_dep_wait();  // the counter and the landing buffers belong to the previous grid until now
  const uint32_t epoch = (uint32_t)*reinterpret_cast<const volatile int*>(p.tp_epoch);
  const int par = (int)(epoch & 1u);
  const uint32_t tag = epoch + 1u;
  const uint32_t t16 = (epoch & 0x7fffu) + 1u;
  const int world = p.tp_world, rank = p.tp_rank;
  const int owner = (int)(blockIdx.x % (unsigned)world);
  const bool rsag = p.tp_rsag != 0;
  const bool recv = rsag && owner != rank;
  for (int idx = tid; idx < M * F; idx += nthreads) {
    const int n = idx / F, f = idx % F;
    const int col = f0 + f;
    if (col >= p.N) continue;
    float v = 0.f;
    for (int w = 0; w < nwarps; ++w) v += red[(w * MT + n) * F + f];
    const int64_t o = (int64_t)par * p.tp_half + ((int64_t)rank * p.tp_rows + n) * p.N + col;
    if (rsag)
      st_tagged_sys(p.tp_land[owner] + o, v, tag);
    else
      for (int d = 0; d < world; ++d) st_tagged_sys(p.tp_land[d] + o, v, tag);
  }
  uint64_t t0 = 0;
  bool ok = true;
  uint16_t* y = static_cast<uint16_t*>(p.y);
  for (int idx = tid; ok && idx < M * F; idx += nthreads) {
    const int n = idx / F, f = idx % F;
    const int col = f0 + f;
    if (col >= p.N) continue;
    uint16_t out;
    if (recv) {
      const uint32_t* wp = p.tp_final[rank] + (int64_t)par * p.tp_fhalf + (int64_t)n * p.N + col;
      uint32_t w = ld_word_sys(wp);
      while ((w >> 16) != t16) {
        if (t0 == 0) {
          t0 = globaltimer_ns();
        } else if (globaltimer_ns() - t0 > AWQB_WAIT_TIMEOUT_NS) {
          ok = false;
          break;
        }
        w = ld_word_sys(wp);
      }
      if (!ok) break;
      out = (uint16_t)(w & 0xffffu);
    } else {
      // every rank's word of this value in flight at once, then the laggards
      const uint2* land = p.tp_land[rank] + (int64_t)par * p.tp_half + (int64_t)n * p.N + col;
      const int64_t rstride = (int64_t)p.tp_rows * p.N;
      uint2 w[8];
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < world) w[r] = ld_tagged_sys(land + r * rstride);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r >= world) break;
        while (w[r].y != tag) {
          if (t0 == 0) {
            t0 = globaltimer_ns();
          } else if (globaltimer_ns() - t0 > AWQB_WAIT_TIMEOUT_NS) {
            ok = false;
            break;
          }
          w[r] = ld_tagged_sys(land + r * rstride);
        }
      }
      if (!ok) break;
      float v = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < world) v += __uint_as_float(w[r].x);  // rank order
      if (p.bias != nullptr) v += Tr::to_f32(reinterpret_cast<const uint16_t*>(p.bias)[col]);
      out = Tr::from_f32(v);
      if (rsag) {
        const uint32_t w = (uint32_t)out | (t16 << 16);
        const int64_t fo = (int64_t)par * p.tp_fhalf + (int64_t)n * p.N + col;
        for (int d = 0; d < world; ++d)
          if (d != rank) st_word_sys(p.tp_final[d] + fo, w);
      }
    }
    y[(int64_t)n * p.ldy + col] = out;
  }
  if (!ok) atomicOr(p.err, 8u);  // kErrWaitEpilogue (awqb_gemm.cuh)
  named_bar_sync(1, nthreads);
  if (tid == 0) {
    // The last CTA to finish advances this rank's call counter (the parity of
    // the next fused call). Every CTA read the counter before it counted
    // itself done, and the next kernel reads it after the grid boundary, so
    // no fence is needed (one after the stores to peer memory would wait for
    // their acknowledgements over NVLink).
    if (atomicAdd(p.tp_epoch + 1, 1) == (int)gridDim.x - 1) {
      p.tp_epoch[1] = 0;
      atomicAdd(p.tp_epoch, 1);
    }
  }
}

// Tensor maps (built on the host, awqb_gemm.cu):
//   tm_w: u32 {512 words of a quarter, 4 quarters, KB blocks, NT tiles}, box {4F, 4, W, 1}
//   tm_s: u16 {128 features, GPB groups, KB, NT},                        box {F, GPB, W, 1}
//   tm_z: u32 {16 words, GPB groups, KB, NT},                            box {kZWords, GPB, W, 1}
//   tm_x: u16 {32 k, M rows, K / 32 chunks},                             box {32, M, 4 W}
template <typename T, int F, int MT, int GPB, int W>
__global__ void __launch_bounds__(GemvCfg<F, MT, GPB, W>::kThreads, F == 16 ? 2 : 1)
awq_gemv_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_x,
                const __grid_constant__ GemvParams p) {
  using Cfg = GemvCfg<F, MT, GPB, W>;
  using Tr = GemvTraits<T>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base: barriers first, then the ring.
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - smem_u32(smem_raw));
  const uint32_t bar_full = base;                 // ring x 8 B
  const uint32_t bar_empty = base + 16 * 8;       // ring x 8 B
  const uint32_t ring0 = base + 256;
  const int sbytes = Cfg::stage_bytes(p.M);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ring = p.ring;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(bar_full + 8 * i, 1);
      mbar_init(bar_empty + 8 * i, Cfg::kWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // The next kernel in the stream may be scheduled now: it only prefetches
  // its weights until this grid has finished.
  grid_dep_launch();

  const int f0 = blockIdx.x * F;        // first output feature of this CTA
  const int nt = f0 >> 7;               // 128-feature tile of the blob
  const int r0 = f0 & 127;              // first row inside the tile

  if (warp == Cfg::kWarps) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_s);
      prefetch_tmap(&tm_z);
      prefetch_tmap(&tm_x);
      const uint64_t pol_w = policy_evict_first();   // each weight byte is read once
      const uint64_t pol_x = policy_evict_last();    // every CTA reads the same activations
      const int zc0 = Cfg::kZWords == F / 8 ? (r0 >> 3) : ((r0 >> 3) & ~3);
      const uint32_t tx = Cfg::kWeightTx + (uint32_t)Cfg::x_bytes(p.M);
      const int n_pre = p.stages < ring ? p.stages : ring;
      auto load_weights = [&](int s, uint32_t st, uint32_t fb) {
        tma_load_4d(st, &tm_w, r0 * 4, 0, s * Cfg::kSB, nt, fb, pol_w);
        tma_load_4d(st + Cfg::kSOff, &tm_s, r0, 0, s * Cfg::kSB, nt, fb, pol_w);
        tma_load_4d(st + Cfg::kZOff, &tm_z, zc0, 0, s * Cfg::kSB, nt, fb, pol_w);
      };
      auto load_x = [&](int s, uint32_t st, uint32_t fb) {
        tma_load_3d(st + Cfg::kXOff, &tm_x, 0, 0, s * Cfg::kSB * 4, fb, pol_x);
      };
      for (int s = 0; s < n_pre; ++s) {
        const uint32_t st = ring0 + (uint32_t)(s * sbytes);
        mbar_arrive_expect_tx(bar_full + 8 * s, tx);
        load_weights(s, st, bar_full + 8 * s);
      }
      grid_dep_wait();  // activations may be the previous kernel's output
      for (int s = 0; s < n_pre; ++s) load_x(s, ring0 + (uint32_t)(s * sbytes), bar_full + 8 * s);
      int issued = n_pre;
      bool ok = true;
      for (int s = n_pre; s < p.stages; ++s) {
        const int slot = s % ring;
        const uint32_t phase = (uint32_t)((s / ring) - 1) & 1u;
        if (!mbar_wait(bar_empty + 8 * slot, phase)) {
          atomicOr(p.err, kErrGemvEmpty);
          ok = false;
          break;
        }
        issued = s + 1;
        const uint32_t st = ring0 + (uint32_t)(slot * sbytes);
        mbar_arrive_expect_tx(bar_full + 8 * slot, tx);
        load_weights(s, st, bar_full + 8 * slot);
        load_x(s, st, bar_full + 8 * slot);
      }
      if (!ok) {
        // Leave only once the copies already issued have landed (bounded).
        for (int s = issued - ring < 0 ? 0 : issued - ring; s < issued; ++s) {
          mbar_wait(bar_full + 8 * (s % ring), (uint32_t)(s / ring) & 1u);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ compute warps
  const int g = lane >> 2;
  const int t = lane & 3;
  // Two or four token groups: the zero point is subtracted from every weight
  // pair (four 16-bit subtractions per word) instead of the all-ones MMA,
  // which would add one tensor-pipe MMA per token group and weight MMA pair:
  // the tensor pipe, not the integer pipe, is the bound there.
  constexpr bool kSubZ = MT >= 16;
  float acc[Cfg::kRG][Cfg::kTG][4];
#pragma unroll
  for (int i = 0; i < Cfg::kRG; ++i)
#pragma unroll
    for (int j = 0; j < Cfg::kTG; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

  const int M = p.M;
  // ldmatrix row address of this lane: matrix mi = lane / 8 is (quarter
  // offset mi / 2, row half mi % 2), row lane % 8.
  const int mi = lane >> 3;
  const uint32_t lsm_off = (uint32_t)((((mi >> 1) * F) + (mi & 1) * 8 + (lane & 7)) * 16);
  const int zbase = Cfg::kZWords == F / 8 ? 0 : ((r0 >> 3) & 3);
  // Per-warp offsets inside a stage (warp w owns k-block w).
  const uint32_t w_off = (uint32_t)(warp * 4 * F * 16) + lsm_off;
  const uint32_t s_off = Cfg::kSOff + (uint32_t)(warp * GPB * F * 2) + (uint32_t)(g * 2);
  const uint32_t z_off = Cfg::kZOff + (uint32_t)(warp * GPB * Cfg::kZWords * 4) + (uint32_t)(zbase * 4);
  // Activation rows >= M feed only output columns >= M, which are dropped:
  // such lanes read row M - 1 (any finite value will do), so no load is
  // predicated.
  uint32_t x_off[Cfg::kTG];
#pragma unroll
  for (int j = 0; j < Cfg::kTG; ++j) {
    const int n = min(g + 8 * j, M - 1);
    x_off[j] = Cfg::kXOff + (uint32_t)(warp * 4 * M * 64) + (uint32_t)(n * 64 + t * 16);
  }
  const uint32_t x_qstride = (uint32_t)(M * 64);
  constexpr int QG = 4 / GPB;  // quarters (32 k) per group
  int slot = 0;
  uint32_t phase = 0;
  uint32_t st = ring0;
  bool ok = true;
  for (int s = 0; s < p.stages; ++s) {
    if (!mbar_wait(bar_full + 8 * slot, phase)) {
      atomicOr(p.err, kErrGemvFull);
      ok = false;
      break;
    }
    if (s * Cfg::kSB + warp < p.kb_real) {
      // packed words of every row group (rows g / g + 8 of quarters 0..3),
      // the activations of the four quarters, (OFF + z) and scale pairs
      uint32_t wa[Cfg::kRG][4][2];
#pragma unroll
      for (int rg = 0; rg < Cfg::kRG; ++rg)
#pragma unroll
        for (int q = 0; q < 4; q += 2)
          ldsm_x4(st + w_off + (uint32_t)(q * F * 16 + rg * 256), wa[rg][q][0], wa[rg][q][1], wa[rg][q + 1][0],
                  wa[rg][q + 1][1]);
#pragma unroll
      for (int grp = 0; grp < GPB; ++grp) {
        // OFF + z (as a float, or as a 16-bit pair to subtract) and the scales
        // of rows g and g + 8 of every row group
        float oz[Cfg::kRG][2], sc[Cfg::kRG][2];
        uint32_t zz[Cfg::kRG][2];
#pragma unroll
        for (int rg = 0; rg < Cfg::kRG; ++rg)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t zw = lds32(st + z_off + (uint32_t)((grp * Cfg::kZWords + rg * 2 + h) * 4));
            const uint32_t z = (zw >> (4 * g)) & 0xFu;
            if constexpr (kSubZ)
              zz[rg][h] = Tr::zero2(z);
            else
              oz[rg][h] = Tr::kOff + (float)z;
            sc[rg][h] = Tr::to_f32((uint16_t)lds16(st + s_off + (uint32_t)((grp * F + rg * 16 + h * 8) * 2)));
          }
        // one accumulator chain per (row group, token group) for the group,
        // and the activation sums X (all-ones operand A)
        float d[Cfg::kRG][Cfg::kTG][4];
        float xs[Cfg::kTG][4];
#pragma unroll
        for (int qi = 0; qi < QG; ++qi) {
          const int q = grp * QG + qi;
          uint4 xb[Cfg::kTG];
#pragma unroll
          for (int j = 0; j < Cfg::kTG; ++j) xb[j] = lds128(st + x_off[j] + (uint32_t)q * x_qstride);
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            const bool first = qi == 0 && pp == 0;
#pragma unroll
            for (int rg = 0; rg < Cfg::kRG; ++rg) {
              const uint32_t wg = wa[rg][q][0];
              const uint32_t wg8 = wa[rg][q][1];
              uint32_t a0 = nib_pair<Tr::kMagic>(wg, 2 * pp);
              uint32_t a1 = nib_pair<Tr::kMagic>(wg8, 2 * pp);
              uint32_t a2 = nib_pair<Tr::kMagic>(wg, 2 * pp + 1);
              uint32_t a3 = nib_pair<Tr::kMagic>(wg8, 2 * pp + 1);
              if constexpr (kSubZ) {  // q - z, exact
                a0 = Tr::sub2(a0, zz[rg][0]);
                a1 = Tr::sub2(a1, zz[rg][1]);
                a2 = Tr::sub2(a2, zz[rg][0]);
                a3 = Tr::sub2(a3, zz[rg][1]);
              }
#pragma unroll
              for (int j = 0; j < Cfg::kTG; ++j) {
                const uint32_t b0 = pp == 0 ? xb[j].x : xb[j].z;
                const uint32_t b1 = pp == 0 ? xb[j].y : xb[j].w;
                if (first)
                  mma16816_z<T>(d[rg][j], a0, a1, a2, a3, b0, b1);
                else
                  mma16816<T>(d[rg][j], a0, a1, a2, a3, b0, b1);
              }
            }
            if constexpr (!kSubZ) {
#pragma unroll
              for (int j = 0; j < Cfg::kTG; ++j) {
                const uint32_t b0 = pp == 0 ? xb[j].x : xb[j].z;
                const uint32_t b1 = pp == 0 ? xb[j].y : xb[j].w;
                if (first)
                  mma16816_z<T>(xs[j], Tr::kOnes, Tr::kOnes, Tr::kOnes, Tr::kOnes, b0, b1);
                else
                  mma16816<T>(xs[j], Tr::kOnes, Tr::kOnes, Tr::kOnes, Tr::kOnes, b0, b1);
              }
            }
          }
        }
#pragma unroll
        for (int rg = 0; rg < Cfg::kRG; ++rg)
#pragma unroll
          for (int j = 0; j < Cfg::kTG; ++j) {
            if constexpr (kSubZ) {
              // acc += s * D for rows g and g + 8 (D = sum x (q - z))
              acc[rg][j][0] = fmaf(sc[rg][0], d[rg][j][0], acc[rg][j][0]);
              acc[rg][j][1] = fmaf(sc[rg][0], d[rg][j][1], acc[rg][j][1]);
              acc[rg][j][2] = fmaf(sc[rg][1], d[rg][j][2], acc[rg][j][2]);
              acc[rg][j][3] = fmaf(sc[rg][1], d[rg][j][3], acc[rg][j][3]);
            } else {
              // acc += s * (D - (OFF + z) * X) for rows g and g + 8 (X of
              // tokens 2t and 2t + 1 sits in the first two elements of the
              // ones product)
              acc[rg][j][0] = fmaf(sc[rg][0], fmaf(-oz[rg][0], xs[j][0], d[rg][j][0]), acc[rg][j][0]);
              acc[rg][j][1] = fmaf(sc[rg][0], fmaf(-oz[rg][0], xs[j][1], d[rg][j][1]), acc[rg][j][1]);
              acc[rg][j][2] = fmaf(sc[rg][1], fmaf(-oz[rg][1], xs[j][0], d[rg][j][2]), acc[rg][j][2]);
              acc[rg][j][3] = fmaf(sc[rg][1], fmaf(-oz[rg][1], xs[j][1], d[rg][j][3]), acc[rg][j][3]);
            }
          }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * slot);
    st += (uint32_t)sbytes;
    if (++slot == ring) {
      slot = 0;
      phase ^= 1u;
      st = ring0;
    }
  }

  // ------------------------------------------------------------ epilogue
  // All compute warps are past their last stage: the ring holds the
  // cross-warp reduction [warp][token][F] fp32 (the host sizes the ring so
  // that it fits).
  const bool all_ok = named_bar_and(1, 32 * Cfg::kWarps, ok);
  if (!all_ok) return;
  float* red = reinterpret_cast<float*>(base_ptr + 256);
#pragma unroll
  for (int rg = 0; rg < Cfg::kRG; ++rg)
#pragma unroll
    for (int j = 0; j < Cfg::kTG; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int f = rg * 16 + g + (e >> 1) * 8;
        const int n = j * 8 + 2 * t + (e & 1);
        red[(warp * MT + n) * F + f] = acc[rg][j][e];
      }
  named_bar_sync(1, 32 * Cfg::kWarps);
  const T* bias = static_cast<const T*>(p.bias);
  uint16_t* y = static_cast<uint16_t*>(p.y);
  const int tid = threadIdx.x;
  if (p.tp_world > 0) {
    gemv_exchange<T, F, MT>(p, red, f0, Cfg::kWarps);
    return;
  }
  if (!p.silu_mul) {
    for (int idx = tid; idx < M * F; idx += 32 * Cfg::kWarps) {
      const int n = idx / F, f = idx % F;
      const int col = f0 + f;
      if (col >= p.N) continue;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < Cfg::kWarps; ++w) v += red[(w * MT + n) * F + f];
      if (bias != nullptr) v += Tr::to_f32(reinterpret_cast<const uint16_t*>(bias)[col]);
      y[(int64_t)n * p.ldy + col] = Tr::from_f32(v);
    }
  } else {
    for (int idx = tid; idx < M * (F / 2); idx += 32 * Cfg::kWarps) {
      const int n = idx / (F / 2), jj = idx % (F / 2);
      const int f = 2 * jj;
      const int col = f0 + f;
      if (col >= p.N) continue;
      float gv = 0.f, uv = 0.f;
#pragma unroll
      for (int w = 0; w < Cfg::kWarps; ++w) {
        gv += red[(w * MT + n) * F + f];
        uv += red[(w * MT + n) * F + f + 1];
      }
      if (bias != nullptr) {
        gv += Tr::to_f32(reinterpret_cast<const uint16_t*>(bias)[col]);
        uv += Tr::to_f32(reinterpret_cast<const uint16_t*>(bias)[col + 1]);
      }
      // silu(g) = g * sigmoid(g), sigmoid(g) = 0.5 * (1 + tanh(g / 2))
      float th;
      asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(0.5f * gv));
      const float v = gv * (0.5f + 0.5f * th) * uv;
      y[(int64_t)n * p.ldy + (col >> 1)] = Tr::from_f32(v);
    }
  }
}

}  // namespace awqb
