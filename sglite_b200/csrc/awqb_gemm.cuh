// W4A16 GEMM for sm_100a: Y[M, N] = X[M, K] * dequant(blob)[K, N].
//
// One kernel serves decode (M <= 64), mid-size and prefill batches, and the MoE
// grouped variant. It replaces the reference's awq_gemm_kernel
// (layers/quantization/awq_triton.py:16-136) and Marlin's gptq_marlin_gemm
// (marlin_utils.py:388-410).
//
// Tile: 128 output features (MMA M, operand A = dequantised weights, K-major)
//       x NTOK tokens (MMA N, operand B = activations, K-major), fp32
//       accumulator in TMEM. One pipeline stage is 128 input features.
//
// Warp roles (14 warps):
//   warp 0        producer: bulk copy of the packed weight block + two TMA
//                 tile loads of X per stage (128-byte swizzle).
//   warp 1        TMEM allocator and single-thread tcgen05.mma issuer.
//   warps 2..5    epilogue: tcgen05.ld of the accumulator, bias, store (or
//                 split-K partials and the fix-up of the last contributor).
//   warps 6..13   dequantisers: packed int4 in shared memory -> fp16/bf16 tile
//                 in the UMMA 128-byte-swizzle K-major layout.
//
// Work partition (stream-K): the (tile, k-block) units of the whole problem are
// split evenly over the persistent CTAs; a CTA walks its units as segments,
// one per tile it touches. A tile covered by a single CTA is stored directly;
// a tile shared by several CTAs is reduced by whichever contributor finishes
// last (an atomic counter per tile; nobody waits), summing the partials in
// contributor order so the result is deterministic. The accumulator is double
// buffered in TMEM so the epilogue of one segment overlaps the next mainloop.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "awqb_layout.cuh"
#include "awqb_ptx.cuh"

namespace awqb {

template <typename T> struct IsBf16 { static constexpr bool value = false; };
template <> struct IsBf16<__nv_bfloat16> { static constexpr bool value = true; };

__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }
__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }
__host__ __device__ constexpr int pow2ceil(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Error bits written by kernels when a bounded wait gives up.
enum DeviceError : uint32_t {
  kErrWaitProducer = 1u,
  kErrWaitMma = 2u,
  kErrWaitDequant = 4u,
  kErrWaitEpilogue = 8u,
  kErrWaitDrain = 16u,
};

struct GemmParams {
  const uint8_t* blob;          // weights; grouped: base of [E][blob_stride]
  int64_t blob_stride;          // grouped: bytes between experts' blobs
  const int32_t* tile_expert;   // grouped: expert id per m-tile, else null
  const int32_t* rows_valid;    // grouped: device count of rows in use, else null
  const void* bias;             // [N] activation dtype, or null
  void* y;                      // output rows of ldy elements
  int64_t ldy;
  const int32_t* row_map;       // if set: output row = row_map[m] (rows >= num_valid skipped)
  const float* row_scale;       // if set: output *= row_scale[output row]
  int32_t num_valid;            // see row_map
  int32_t M, N, K;
  int32_t NT, KB, MT;           // feature tiles, k-blocks, token tiles (max)
  float* ws_part;               // [gridDim.x][2][128 * NTOK] fp32 partial tiles
  int32_t* ws_cnt;              // [MT * NT] arrival counters, zero between calls
  uint32_t* err;                // device error word
};

template <int NTOK, int GPB>
struct GemmCfg {
  static constexpr int kThreads = 448;
  static constexpr int kEpiWarp0 = 2;
  static constexpr int kNumEpiWarps = 4;
  static constexpr int kDqWarp0 = 6;
  static constexpr int kNumDqWarps = 8;
  static constexpr int kPkBytes = block_bytes_for_gpb(GPB);
  static constexpr int kPkRegion = (kPkBytes + 1023) / 1024 * 1024;
  static constexpr int kXAtom = NTOK * 128;          // 64 k x NTOK rows, 128 B rows
  static constexpr int kXBytes = 2 * kXAtom;
  static constexpr int kLStage = kPkRegion + kXBytes;
  static constexpr int kWStage = 2 * 16384;          // 128 rows x 128 k, two swizzle atoms
  static constexpr int kSD = 2;
  static constexpr int kBudget = 225 * 1024 - 1024 - 512;
  static constexpr int kSL = cmin(12, (kBudget - kSD * kWStage) / kLStage);
  static constexpr int kSmemBytes = 1024 + kSL * kLStage + kSD * kWStage + 512;
  static_assert((2 * kSL + 2 * kSD + 5) * 8 + 16 <= 512, "barrier area overflow");
  static constexpr int kTmemCols = pow2ceil(cmax(32, 2 * NTOK));
  static_assert(kSL >= 2, "not enough shared memory for two load stages");
  static_assert(NTOK % 16 == 0 && NTOK >= 16 && NTOK <= 256, "MMA N must be 16..256 step 16");
  static_assert(kPkBytes % 16 == 0, "bulk copy size must be a multiple of 16");
};

// Owner of unit u when U units are split over C CTAs as [cU/C, (c+1)U/C).
__device__ __forceinline__ int unit_owner(int64_t u, int64_t U, int64_t C) {
  return (int)(((u + 1) * C - 1) / U);
}

template <typename T, int NTOK, int GPB>
__global__ void __launch_bounds__(448, 1)
awq_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmParams p) {
  using Cfg = GemmCfg<NTOK, GPB>;
  using DQ = DqTraits<T>;
  constexpr int SL = Cfg::kSL;
  constexpr int SD = Cfg::kSD;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  uint8_t* lring = base;
  uint8_t* wring = base + SL * Cfg::kLStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(wring + SD * Cfg::kWStage);
  // barrier slots
  uint64_t* full_l = bars;             // [SL]  TMA bytes landed
  uint64_t* empty_l = bars + SL;       // [SL]  dequant warps + MMA done with the stage
  uint64_t* full_d = bars + 2 * SL;    // [SD]  dequantised tile written
  uint64_t* empty_d = full_d + SD;     // [SD]  MMA done reading the tile
  uint64_t* acc_full = empty_d + SD;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* drain = acc_empty + 2;     // [1]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  int* s_flag = const_cast<int*>(reinterpret_cast<volatile int*>(s_tmem + 2));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work partition (identical in every role)
  int MT = p.MT;
  if (p.rows_valid != nullptr) {
    const int rows = *p.rows_valid;
    MT = cmin(MT, (rows + NTOK - 1) / NTOK);
  }
  const int64_t U = (int64_t)MT * p.NT * p.KB;
  // Never more contributors than units, so every CTA below C owns >= 1 unit.
  const int64_t C = (int64_t)gridDim.x < U ? (int64_t)gridDim.x : U;
  const bool has_work = (int64_t)blockIdx.x < C;
  const int64_t u_begin = has_work ? (int64_t)blockIdx.x * U / C : 0;
  const int64_t u_end = has_work ? (int64_t)(blockIdx.x + 1) * U / C : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SL; ++i) {
      mbar_init(smem_u32(&full_l[i]), 1);
      mbar_init(smem_u32(&empty_l[i]), Cfg::kNumDqWarps + 1);
    }
    for (int i = 0; i < SD; ++i) {
      mbar_init(smem_u32(&full_d[i]), Cfg::kNumDqWarps);
      mbar_init(smem_u32(&empty_d[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&acc_full[i]), 1);
      mbar_init(smem_u32(&acc_empty[i]), Cfg::kNumEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    *s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tmap_x);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  if (U == 0 || u_begin >= u_end) {
    // nothing to do for this CTA
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int64_t it = 0;
      for (int64_t u = u_begin; u < u_end; ++u, ++it) {
        const int sl = (int)(it % SL);
        if (it >= SL) {
          if (!mbar_wait(smem_u32(&empty_l[sl]), (uint32_t)((it / SL) - 1) & 1u)) {
            atomicOr(p.err, kErrWaitProducer);
            *s_abort = 1;
            break;
          }
        }
        if (*s_abort) break;
        const int64_t tile = u / p.KB;
        const int kb = (int)(u - tile * p.KB);
        const int mt = (int)(tile / p.NT);
        const int nt = (int)(tile - (int64_t)mt * p.NT);
        const uint8_t* blob = p.blob;
        if (p.tile_expert != nullptr) blob += (int64_t)p.tile_expert[mt] * p.blob_stride;
        const uint8_t* src = blob + ((int64_t)nt * p.KB + kb) * Cfg::kPkBytes;
        uint8_t* st = lring + sl * Cfg::kLStage;
        const uint32_t bar = smem_u32(&full_l[sl]);
        mbar_arrive_expect_tx(bar, Cfg::kPkBytes + Cfg::kXBytes);
        bulk_g2s(smem_u32(st), src, Cfg::kPkBytes, bar, pol_w);
        tma_load_2d(smem_u32(st + Cfg::kPkRegion), &tmap_x, kb * kBlockK, mt * NTOK, bar, pol_x);
        tma_load_2d(smem_u32(st + Cfg::kPkRegion + Cfg::kXAtom), &tmap_x, kb * kBlockK + 64,
                    mt * NTOK, bar, pol_x);
      }
      // Do not leave while copies into this CTA's shared memory are in flight.
      const int64_t issued = it;
      for (int64_t j = (issued > SL ? issued - SL : 0); j < issued; ++j) {
        if (!mbar_wait(smem_u32(&full_l[j % SL]), (uint32_t)(j / SL) & 1u)) {
          atomicOr(p.err, kErrWaitDrain);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, NTOK, IsBf16<T>::value ? 1 : 0);
      int64_t it = 0;
      int seg = 0;
      bool ok = true;
      for (int64_t u = u_begin; u < u_end && ok; ++seg) {
        const int64_t tile = u / p.KB;
        const int64_t seg_end = (tile + 1) * p.KB < u_end ? (tile + 1) * p.KB : u_end;
        const int64_t seg_begin = u;
        const int buf = seg & 1;
        if (seg >= 2) {
          if (!mbar_wait(smem_u32(&acc_empty[buf]), (uint32_t)((seg >> 1) - 1) & 1u)) {
            atomicOr(p.err, kErrWaitMma);
            *s_abort = 1;
            break;
          }
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * NTOK);
        for (; u < seg_end; ++u, ++it) {
          const int sl = (int)(it % SL);
          const int sd = (int)(it % SD);
          if (!mbar_wait(smem_u32(&full_l[sl]), (uint32_t)(it / SL) & 1u) ||
              !mbar_wait(smem_u32(&full_d[sd]), (uint32_t)(it / SD) & 1u)) {
            atomicOr(p.err, kErrWaitMma);
            *s_abort = 1;
            ok = false;
            break;
          }
          if (*s_abort) { ok = false; break; }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(wring + sd * Cfg::kWStage);
          const uint32_t x_addr = smem_u32(lring + sl * Cfg::kLStage + Cfg::kPkRegion);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t koff = (uint32_t)((kk & 3) * 32);
            const uint64_t adesc = make_sw128_kmajor_desc(w_addr + (kk >> 2) * 16384 + koff);
            const uint64_t bdesc = make_sw128_kmajor_desc(x_addr + (kk >> 2) * Cfg::kXAtom + koff);
            tc_mma_f16(d_tmem, adesc, bdesc, idesc, (u != seg_begin || kk > 0) ? 1u : 0u);
          }
          tc_commit(smem_u32(&empty_d[sd]));
          tc_commit(smem_u32(&empty_l[sl]));
        }
        if (ok) tc_commit(smem_u32(&acc_full[buf]));
      }
      // Every MMA issued must finish before TMEM is released.
      tc_commit(smem_u32(drain));
      if (!mbar_wait(smem_u32(drain), 0)) atomicOr(p.err, kErrWaitDrain);
    }
  } else if (warp >= Cfg::kEpiWarp0 && warp < Cfg::kEpiWarp0 + Cfg::kNumEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int f = q * 32 + lane;            // feature row within the tile
    const int etid = threadIdx.x - Cfg::kEpiWarp0 * 32;
    int seg = 0;
    for (int64_t u = u_begin; u < u_end; ++seg) {
      const int64_t tile = u / p.KB;
      const int64_t t_begin = tile * p.KB;
      const int64_t t_end = t_begin + p.KB;
      const int64_t seg_end = t_end < u_end ? t_end : u_end;
      const int buf = seg & 1;
      const int mt = (int)(tile / p.NT);
      const int nt = (int)(tile - (int64_t)mt * p.NT);
      const int n = nt * kBlockN + f;
      int rows_here = p.M - mt * NTOK;
      if (p.rows_valid != nullptr) rows_here = cmin(rows_here, *p.rows_valid - mt * NTOK);
      rows_here = cmax(0, cmin(NTOK, rows_here));
      const int ncols = (rows_here + 15) & ~15;

      if (!mbar_wait(smem_u32(&acc_full[buf]), (uint32_t)(seg >> 1) & 1u)) {
        atomicOr(p.err, kErrWaitEpilogue);
        *s_abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_addr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * NTOK);
      const int c_first = unit_owner(t_begin, U, C);
      const int c_last = unit_owner(t_end - 1, U, C);
      const bool whole = (c_first == c_last);

      float bias_v = 0.f;
      if (p.bias != nullptr && n < p.N) bias_v = (float)reinterpret_cast<const T*>(p.bias)[n];

      if (whole) {
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(t_addr + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int mloc = c0 + c;
            if (mloc < rows_here && n < p.N) {
              int m = mt * NTOK + mloc;
              float val = __uint_as_float(v[c]) + bias_v;
              if (p.row_map != nullptr) {
                m = p.row_map[m];
                if (m >= p.num_valid) continue;
              }
              if (p.row_scale != nullptr) val *= p.row_scale[m];
              reinterpret_cast<T*>(p.y)[(int64_t)m * p.ldy + n] = (T)val;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acc_empty[buf]));
      } else {
        // Partial tile: this CTA's slot 0 holds its first segment, slot 1 its last.
        const int slot = (u == u_begin) ? 0 : 1;
        float* part = p.ws_part + ((int64_t)blockIdx.x * 2 + slot) * (128 * NTOK);
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(t_addr + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 16; ++c) __stcg(&part[(c0 + c) * 128 + f], __uint_as_float(v[c]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acc_empty[buf]));
        __threadfence();
        named_bar_sync(1, Cfg::kNumEpiWarps * 32);
        if (etid == 0) {
          const int prev = atomicAdd(&p.ws_cnt[tile], 1);
          *s_flag = (prev == c_last - c_first) ? 1 : 0;
        }
        named_bar_sync(1, Cfg::kNumEpiWarps * 32);
        const int last = *s_flag;
        named_bar_sync(1, Cfg::kNumEpiWarps * 32);  // s_flag may be rewritten next segment
        if (last) {
          __threadfence();
          for (int mloc = 0; mloc < rows_here; ++mloc) {
            float acc = 0.f;
            for (int c = c_first; c <= c_last; ++c) {
              // tile is contributor c's first segment iff c's range starts inside it
              const int64_t cb = (int64_t)c * U / C;
              const int cs = (cb >= t_begin) ? 0 : 1;
              acc += __ldcg(&p.ws_part[((int64_t)c * 2 + cs) * (128 * NTOK) + mloc * 128 + f]);
            }
            if (n < p.N) {
              int m = mt * NTOK + mloc;
              float val = acc + bias_v;
              if (p.row_map != nullptr) {
                m = p.row_map[m];
                if (m >= p.num_valid) continue;
              }
              if (p.row_scale != nullptr) val *= p.row_scale[m];
              reinterpret_cast<T*>(p.y)[(int64_t)m * p.ldy + n] = (T)val;
            }
          }
          if (etid == 0) p.ws_cnt[tile] = 0;
        }
      }
      u = seg_end;
    }
    tc_fence_before();
  } else if (warp >= Cfg::kDqWarp0) {
    // ------------------------------------------------------------ dequantisers
    const int d = threadIdx.x - Cfg::kDqWarp0 * 32;  // 0..255
    const int r = d & 127;                           // weight row (feature) in the tile
    const int h = d >> 7;                            // which 64-wide half of the stage
    const int rsw = r & 7;
    int64_t it = 0;
    for (int64_t u = u_begin; u < u_end; ++u, ++it) {
      const int sl = (int)(it % SL);
      const int sd = (int)(it % SD);
      if (!mbar_wait(smem_u32(&full_l[sl]), (uint32_t)(it / SL) & 1u)) {
        atomicOr(p.err, kErrWaitDequant);
        *s_abort = 1;
        break;
      }
      if (it >= SD) {
        if (!mbar_wait(smem_u32(&empty_d[sd]), (uint32_t)((it / SD) - 1) & 1u)) {
          atomicOr(p.err, kErrWaitDequant);
          *s_abort = 1;
          break;
        }
      }
      if (*s_abort) break;
      const uint8_t* pk = lring + sl * Cfg::kLStage;
      uint8_t* wt = wring + sd * Cfg::kWStage + h * 16384 + r * 128;
      typename DQ::Terms terms[GPB >= 4 ? 2 : 1];
      {
        uint16_t sb;
        uint32_t z;
        if constexpr (GPB >= 4) {
          block_scale_zero(pk, GPB, 2 * h, r, sb, z);
          terms[0] = DQ::make(sb, z);
          block_scale_zero(pk, GPB, 2 * h + 1, r, sb, z);
          terms[1] = DQ::make(sb, z);
        } else {
          block_scale_zero(pk, GPB, GPB == 2 ? h : 0, r, sb, z);
          terms[0] = DQ::make(sb, z);
        }
      }
#pragma unroll
      for (int jq = 0; jq < 2; ++jq) {
        const int j4 = 2 * h + jq;
        const uint4 v = *reinterpret_cast<const uint4*>(pk + ((j4 * 128 + r) << 4));
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jl = jq * 4 + e;  // word index within this half: 0..7
          const uint4 o = DQ::dq8(wv[e], terms[GPB >= 4 ? jq : 0]);
          *reinterpret_cast<uint4*>(wt + ((jl ^ rsw) << 4)) = o;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&full_d[sd]));
        mbar_arrive(smem_u32(&empty_l[sl]));
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace awqb
