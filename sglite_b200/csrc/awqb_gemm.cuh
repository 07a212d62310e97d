// W4A16 GEMM for sm_100a: Y[M, N] = X[M, K] * dequant(blob)[K, N].
//
// One kernel serves decode (M <= 64), mid-size and prefill batches, and the MoE
// grouped variant. It replaces the reference's awq_gemm_kernel
// (layers/quantization/awq_triton.py:16-136) and Marlin's gptq_marlin_gemm
// (marlin_utils.py:388-410).
//
// Tile: 128 output features (MMA M, operand A = dequantised weights, K-major)
//       x NTOK tokens (MMA N, operand B = activations, K-major), fp32
//       accumulator in TMEM. One pipeline stage is kSB blocks of 128 input
//       features: 256 for token tiles <= 64, 128 for larger token tiles.
//
// Warp roles (22 warps):
//   warp 0        producer: one bulk copy of the stage's packed weight blocks
//                 (contiguous in the blob) + one 3-D TMA tile load of X per
//                 stage (128-byte swizzle).
//   warp 1        TMEM allocator and single-thread tcgen05.mma issuer.
//   warps 2..5    epilogue: tcgen05.ld of the accumulator, bias, store (or
//                 split-K partials and the fix-up of the last contributor).
//   warps 6..21   dequantisers: packed int4 in shared memory -> fp16/bf16 rows
//                 written straight into tensor memory (tcgen05.st) as the MMA's
//                 A operand (token tiles <= 128), or into shared memory in the
//                 128-byte-swizzle K-major layout (token tile 256, whose
//                 accumulators fill TMEM). Keeping the dequantised weights out
//                 of shared memory is what lets decode stream at HBM speed:
//                 the write + MMA read of a smem copy would cost 4 bytes of
//                 shared-memory bandwidth per weight.
//
// Work partition (Sched): persistent CTAs take whole tiles round-robin while at
// least two full waves remain (neighbouring CTAs share activations in L2), then
// the (tile, stage) units of the last waves are split evenly over the CTAs
// (stream-K); a CTA walks its units as segments, one per tile it touches. A
// tile covered by a single CTA is stored directly;
// a tile shared by several CTAs is reduced by the contributor that arrives last
// (an arrival ticket per tile): it keeps its own partial in TMEM and waits only
// for peers that have already arrived to publish theirs, summing the partials
// in contributor order so the result is deterministic. The accumulator is
// double buffered in TMEM so the epilogue of one segment overlaps the next
// mainloop.
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
  float* ws_part;               // [gridDim.x][2][128 rows][NTOK] fp32 partial tiles
  int32_t* ws_cnt;              // [gridDim.x][2] arrived / published counters of the split tile
                                //   each CTA owns; zero between calls
  uint32_t* err;                // device error word
  int32_t x3d;                  // X tensor map is 3-D {64, rows, K/64}: one load per stage
  int32_t silu_mul;             // columns interleaved gate j, up j: the output is
                                //   silu(gate) * up, N / 2 features, dense rows
  int32_t group_m;              // token tiles per raster group (>= 1)
  int32_t cluster_s;            // >= 2: launched in clusters of cluster_s CTAs, one tile per
                                //   cluster; its partials are reduced through DSMEM
  // Fused all-reduce across tensor-parallel ranks (tp_world >= 2, or 1 to run
  // the exchange against itself): every final value goes as an 8-byte {fp32,
  // call tag} word into every rank's landing buffer; each rank waits for the
  // tp_world words of each of its values and sums them in rank order.
  int32_t tp_world, tp_rank;
  int32_t tp_rows;              // landing rows per slot (>= M)
  int64_t tp_half;              // words per parity half of a landing buffer
  uint2* tp_land[8];            // per rank (peer-mapped): landing words, [2][world][rows][N]
  int32_t* tp_epoch;            // this rank's call counter (tag = epoch + 1, buffer = epoch & 1)
                                //   and the count of CTAs done with the call
  // Reduce-scatter + all-gather mode (tp_rsag): the values of feature tile nt
  // go only to rank nt % world, which sums them, stores them and sends the
  // final values ({16-bit value, 16-bit tag} words) to the other ranks.
  int32_t tp_rsag;
  uint32_t* tp_final[8];        // per rank (peer-mapped): final words, [2][rows][N]
  int64_t tp_fhalf;             // final words per parity half
};

template <int NTOK, int GPB>
struct GemmCfg {
  static constexpr int kEpiWarp0 = 2;
  static constexpr int kNumEpiWarps = 4;
  static constexpr int kDqWarp0 = 6;
  static constexpr int kNumDqWarps = 16;              // two groups of 8
  static constexpr int kDqGroupWarps = 8;
  static constexpr int kThreads = 32 * (kDqWarp0 + kNumDqWarps);
  static constexpr bool kATmem = NTOK <= 128;         // operand A (weights) in tensor memory
  // 128-k blocks per pipeline stage: 256 k for small token tiles (fewer
  // barrier round trips per weight byte), 128 k above so that five stages of
  // activations fit in shared memory.
  static constexpr int kSB = NTOK <= 64 ? 2 : 1;
  static constexpr int kDqPerStage = 8;                 // one group of warps dequantises a stage
  static constexpr int kPkBytes = block_bytes_for_gpb(GPB);   // one packed block
  static constexpr int kPkStage = kSB * kPkBytes;             // bytes of one stage's bulk copy
  static constexpr int kPkRegion = (kPkStage + 1023) / 1024 * 1024;
  static constexpr int kXAtom = NTOK * 128;           // 64 k x NTOK rows, 128 B rows
  static constexpr int kXAtoms = 2 * kSB;
  static constexpr int kXBytes = kXAtoms * kXAtom;
  static constexpr int kLStage = kPkRegion + kXBytes;
  static constexpr int kWStage = kATmem ? 0 : 2 * 16384;  // smem copy of A: 128 rows x 128 k
  static constexpr int kAStageCols = 64 * kSB;         // TMEM columns of one A stage
  static constexpr int kBudget = 225 * 1024 - 1024 - 512;
  static constexpr int kSD = kATmem ? cmin(4, (512 - 2 * NTOK) / kAStageCols) : 2;
  static constexpr int kSL = cmin(16, (kBudget - kSD * kWStage) / kLStage);
  // Scattered output (MoE): each epilogue warp's copy of the tile's destination
  // rows and scales, {row or -1, scale bits} per token row.
  static constexpr int kRowBytes = kNumEpiWarps * NTOK * 8;
  static constexpr int kSmemBytes = 1024 + kSL * kLStage + kSD * kWStage + 512 + kRowBytes;
  static constexpr int kAcol0 = 2 * NTOK;             // TMEM: [0, 2*NTOK) accumulators, then A stages
  static constexpr int kTmemCols = pow2ceil(cmax(32, 2 * NTOK + (kATmem ? kSD * kAStageCols : 0)));
  static_assert(kSD >= 2, "need two A stages");
  static_assert(kTmemCols <= 512, "TMEM over capacity");
  static_assert((3 * kSL + 2 * kSD + 6) * 8 + 32 <= 512, "barrier area overflow");
  static_assert(kSL >= 2, "not enough shared memory for two load stages");
  static_assert(kSmemBytes <= 232448, "shared memory over the sm_100 per-CTA limit");
  static_assert(NTOK % 16 == 0 && NTOK >= 16 && NTOK <= 256, "MMA N must be 16..256 step 16");
  static_assert(kPkBytes % 16 == 0, "bulk copy size must be a multiple of 16");
};

// Ring slot + phase bit, advanced without divisions.
struct RingPos {
  int idx = 0;
  uint32_t phase = 0;
  template <int S>
  __device__ __forceinline__ void next() {
    if (++idx == S) {
      idx = 0;
      phase ^= 1u;
    }
  }
};

// Work of one CTA, as a sequence of "local" units j = 0 .. n_local-1 (a unit is
// one pipeline stage of one tile; tile t maps to (mt, nt) by tile_mn).
//  * Data-parallel phase, while at least two full waves of tiles remain: whole
//    tiles c, c + C, c + 2C, ... Concurrent CTAs work on neighbouring tiles, so
//    they share activation rows (and weights) in L2.
//  * Stream-K phase over the units of the last one to two waves, split evenly
//    into contiguous ranges [c U_sk / C, (c+1) U_sk / C). Tiles cut by a range
//    boundary are reduced across their contributors (see the epilogue).
// Decode-sized problems (fewer tiles than two waves) are stream-K only.
struct Sched {
  int KBS, NT, MT, C, c;
  int GM;        // token tiles per raster group
  int dp_units;  // units of this CTA's data-parallel tiles
  int sk_base;   // first global unit of the stream-K phase (a tile boundary)
  int U_sk;      // units in the stream-K phase (>= C)
  int sk_begin;  // this CTA's stream-K range start, relative to sk_base
  int n_local;   // units this CTA processes (0 for CTAs >= C)
  __device__ __forceinline__ void init(int MT_, int KBS_, int NT_, int GM_, int grid, int cta) {
    KBS = KBS_;
    NT = NT_;
    MT = MT_;
    GM = GM_ > 0 ? GM_ : 1;
    const int T = MT * NT;
    const int U = T * KBS;
    C = grid < U ? grid : U;  // never more CTAs than units: each CTA below C has work
    c = cta;
    const int waves = T / C;
    const int n_dp = waves >= 2 ? waves - 1 : 0;
    dp_units = n_dp * KBS;
    sk_base = n_dp * C * KBS;
    U_sk = U - sk_base;
    if (cta >= C) {
      dp_units = 0;
      sk_begin = 0;
      n_local = 0;
      return;
    }
    sk_begin = sk_start(cta);
    n_local = dp_units + sk_start(cta + 1) - sk_begin;
  }
  // Stream-K: first unit (relative) of contributor cj, and the owner of unit r.
  // U_sk < 2 C KBS, so the products stay below 2 C^2 KBS < 2^31 (checked by
  // the host) and 32-bit unsigned arithmetic suffices.
  __device__ __forceinline__ int sk_start(int cj) const { return (int)((unsigned)cj * (unsigned)U_sk / (unsigned)C); }
  __device__ __forceinline__ int sk_owner(int r) const {
    return (int)(((unsigned)r * (unsigned)C + (unsigned)C - 1u) / (unsigned)U_sk);
  }
  // Global unit of local unit j in the stream-K phase.
  __device__ __forceinline__ int sk_global(int j) const { return sk_base + sk_begin + (j - dp_units); }
  // Raster: tiles run through groups of GM token tiles; inside a group the
  // token tile varies fastest, so concurrent CTAs share feature tiles (weights
  // read from DRAM once for up to GM token tiles) and a narrow band of
  // activation rows. GM = 1 walks all feature tiles of one token tile first.
  __device__ __forceinline__ void tile_mn(int t, int& mt, int& nt) const {
    const int gsz = GM * NT;
    const int g = t / gsz;
    const int w = t - g * gsz;
    const int m0 = g * GM;
    const int gm = MT - m0 < GM ? MT - m0 : GM;
    nt = w / gm;
    mt = m0 + (w - nt * gm);
  }
  __device__ __forceinline__ int tile_of(int j) const {
    return j < dp_units ? c + (j / KBS) * C : sk_global(j) / KBS;
  }
  // End (exclusive, local) of the segment - the run of units of one tile - holding j.
  __device__ __forceinline__ int seg_end(int j) const {
    if (j < dp_units) return (j / KBS + 1) * KBS;
    const int g = sk_global(j);
    const int e = j + ((g / KBS + 1) * KBS - g);
    return e < n_local ? e : n_local;
  }
};

// Walks a CTA's local units: stage kb, tile and its (mt, nt); divisions only
// at tile boundaries.
struct WorkPos {
  int j, kb, tile, nt, mt;
  __device__ __forceinline__ void set_tile(int t, const Sched& s) {
    tile = t;
    s.tile_mn(t, mt, nt);
  }
  __device__ __forceinline__ void init(int j0, const Sched& s) {
    j = j0;
    if (j0 < s.dp_units) {
      const int w = j0 / s.KBS;
      kb = j0 - w * s.KBS;
      set_tile(s.c + w * s.C, s);
    } else {
      const int g = s.sk_global(j0);
      const int t = g / s.KBS;
      kb = g - t * s.KBS;
      set_tile(t, s);
    }
  }
  __device__ __forceinline__ void next(const Sched& s) {
    ++j;
    if (j == s.dp_units) {  // into the stream-K range, which may start mid-tile
      init(j, s);
      return;
    }
    if (++kb == s.KBS) {
      kb = 0;
      set_tile(j < s.dp_units ? tile + s.C : tile + 1, s);
    }
  }
};

// silu(g) = g * sigmoid(g) = 0.5 g (1 + tanh(g / 2)), with the hardware tanh
// approximation (relative error ~2^-11, far below the output's bf16 / fp16
// rounding): one special-function instruction instead of exp + reciprocal.
__device__ __forceinline__ float silu_fast(float g) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * g));
  return 0.5f * g * (1.f + t);
}

// Fused all-reduce: one final value, as a tagged word, to every rank's landing
// buffer (out of line: keeps the epilogue's registers free).
__device__ __noinline__ void tp_put(uint2* const* lands, int world, int64_t off, float v, uint32_t tag) {
  for (int d = 0; d < world; ++d) st_tagged_sys(lands[d] + off, v, tag);
}

// Tag of the final words: 15 bits of the call counter, never 0 (a zeroed buffer
// never matches).
__device__ __forceinline__ uint32_t tp_tag16(uint32_t epoch) { return (epoch & 0x7fffu) + 1u; }

// Fused all-reduce at the end of a cluster split-K tile: this CTA's slice,
// features n0 .. n0+nf-1 of rows m0 .. m0+rows-1, was sent to the landing
// buffers. Wait for the tagged words, then store (sum of every rank's partial
// in rank order, or, in the reduce-scatter mode on a rank that does not own the
// tile, the owner's final values; the owner sends those). Out of line: runs
// once per CTA.
template <typename T>
__device__ __noinline__ void tp_cluster_finish(const GemmParams& p, int n0, int nf, int m0, int rows,
                                               uint32_t epoch) {
  const int par = (int)(epoch & 1u);
  const uint32_t tag = epoch + 1u;
  const uint32_t t16 = tp_tag16(epoch);
  const bool recv = p.tp_rsag && (n0 / kBlockN) % p.tp_world != p.tp_rank;
  const uint2* land = p.tp_land[p.tp_rank] + (int64_t)par * p.tp_half;
  const uint32_t* fin = p.tp_final[p.tp_rank] + (int64_t)par * p.tp_fhalf;
  uint64_t t0 = 0;
  for (int e = threadIdx.x; e < nf * rows; e += blockDim.x) {
    const int c = e / nf;
    const int n = n0 + (e - c * nf);
    if (n >= p.N) continue;
    const int m = m0 + c;
    T out;
    if (recv) {
      const uint32_t* wp = fin + (int64_t)m * p.N + n;
      uint32_t w = ld_word_sys(wp);
      while ((w >> 16) != t16) {
        if (t0 == 0) {
          t0 = globaltimer_ns();
        } else if (globaltimer_ns() - t0 > AWQB_WAIT_TIMEOUT_NS) {
          atomicOr(p.err, 8u);  // kErrWaitEpilogue
          return;
        }
        w = ld_word_sys(wp);
      }
      const uint16_t b = (uint16_t)(w & 0xffffu);
      out = *reinterpret_cast<const T*>(&b);
    } else {
      // every rank's word of this value in flight at once, then the laggards
      const uint2* wp = land + (int64_t)m * p.N + n;
      const int64_t rstride = (int64_t)p.tp_rows * p.N;
      uint2 w[8];
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < p.tp_world) w[r] = ld_tagged_sys(wp + r * rstride);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r >= p.tp_world) break;
        while (w[r].y != tag) {
          if (t0 == 0) {
            t0 = globaltimer_ns();
          } else if (globaltimer_ns() - t0 > AWQB_WAIT_TIMEOUT_NS) {
            atomicOr(p.err, 8u);
            return;
          }
          w[r] = ld_tagged_sys(wp + r * rstride);
        }
      }
      float v = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < p.tp_world) v += __uint_as_float(w[r].x);  // rank order
      if (p.bias != nullptr) v += (float)reinterpret_cast<const T*>(p.bias)[n];
      out = (T)v;
      if (p.tp_rsag) {
        const uint32_t w = (uint32_t) * reinterpret_cast<const uint16_t*>(&out) | (t16 << 16);
        const int64_t fo = (int64_t)par * p.tp_fhalf + (int64_t)m * p.N + n;
        for (int d = 0; d < p.tp_world; ++d)
          if (d != p.tp_rank) st_word_sys(p.tp_final[d] + fo, w);
      }
    }
    reinterpret_cast<T*>(p.y)[(int64_t)m * p.ldy + n] = out;
  }
}

// Fused all-reduce, final step for one feature column of a tile: wait until
// each of the world ranks' words for rows 0..rows-1 carries this call's tag,
// sum them in rank order, add the bias and store. land points at rank 0's word
// of row 0 (slots are rows_cap * ld words apart); bounded wait.
template <typename T>
__device__ __forceinline__ void tp_finalize_column(const uint2* land, T* y, int64_t ldy, int ld, int rows_cap,
                                                int world, int rows, float bias, uint32_t tag, uint32_t* err) {
  // 8 words in flight: rows_per = 8 / world rows per batch, each with all
  // world ranks' words, summed in rank order.
  const int rows_per = world >= 8 ? 1 : 8 / world;
  uint64_t t0 = 0;
  for (int c0 = 0; c0 < rows; c0 += rows_per) {
    uint2 w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int cr = i / world;
      const int r = i - cr * world;
      const bool live = cr < rows_per && c0 + cr < rows;
      w[i] = live ? ld_tagged_sys(land + ((int64_t)r * rows_cap + c0 + cr) * ld) : make_uint2(0u, tag);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (w[i].y == tag) continue;
      const int cr = i / world;
      const int r = i - cr * world;
      const uint2* wp = land + ((int64_t)r * rows_cap + c0 + cr) * ld;
      do {
        if (t0 == 0) {
          t0 = globaltimer_ns();
        } else if (globaltimer_ns() - t0 > AWQB_WAIT_TIMEOUT_NS) {
          atomicOr(err, 8u);  // kErrWaitEpilogue
          return;
        }
        w[i] = ld_tagged_sys(wp);
      } while (w[i].y != tag);
    }
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int cr = i / world;
      const int r = i - cr * world;
      if (cr >= rows_per || c0 + cr >= rows) break;
      v += __uint_as_float(w[i].x);
      if (r == world - 1) {
        y[(int64_t)(c0 + cr) * ldy] = (T)(v + bias);
        v = 0.f;
      }
    }
  }
}

template <typename T, int NTOK, int GPB>
__global__ void __maxnreg__(80)
awq_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<NTOK, GPB>;
  using DQ = DqTraits<T>;
  constexpr int SL = Cfg::kSL;
  constexpr int SD = Cfg::kSD;
  constexpr int SB = Cfg::kSB;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  uint8_t* lring = base;
  uint8_t* wring = base + SL * Cfg::kLStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(wring + SD * Cfg::kWStage);
  uint64_t* full_w = bars;             // [SL]  the stage's packed weights landed
  uint64_t* full_x = bars + SL;        // [SL]  the stage's activations landed
  uint64_t* empty_l = bars + 2 * SL;   // [SL]  dequant warps + MMA done with the stage
  uint64_t* full_d = bars + 3 * SL;    // [SD]  dequantised A stage written
  uint64_t* empty_d = full_d + SD;     // [SD]  MMA done reading the A stage
  uint64_t* acc_full = empty_d + SD;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* drain = acc_empty + 2;     // [1]
  uint64_t* red_bar = drain + 1;       // [1]  peers' partials landed (bulk-copy reduction)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(red_bar + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile int* s_flag = reinterpret_cast<volatile int*>(s_tmem + 2);  // [2]
  volatile uint32_t* s_tpe = s_tmem + 4;  // fused all-reduce: this call's counter value
  int2* row_slots = reinterpret_cast<int2*>(reinterpret_cast<uint8_t*>(bars) + 512);  // [epi warp][NTOK]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work partition (identical in every role; all 32-bit, units < 2^31)
  int MT = p.MT;
  if (p.rows_valid != nullptr) {
    const int rows = *p.rows_valid;
    MT = cmin(MT, (rows + NTOK - 1) / NTOK);
  }
  const int KB = p.KB, NT = p.NT;
  const int KBS = KB / SB;  // stages per tile (KB is even)
  Sched sch;
  sch.init(MT, KBS, NT, p.group_m, (int)gridDim.x, (int)blockIdx.x);
  const int n_local = sch.n_local;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SL; ++i) {
      mbar_init(smem_u32(&full_w[i]), 1);
      mbar_init(smem_u32(&full_x[i]), 1);
      mbar_init(smem_u32(&empty_l[i]), Cfg::kDqPerStage + 1);
    }
    for (int i = 0; i < SD; ++i) {
      mbar_init(smem_u32(&full_d[i]), Cfg::kDqPerStage);
      mbar_init(smem_u32(&empty_d[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&acc_full[i]), 1);
      mbar_init(smem_u32(&acc_empty[i]), Cfg::kNumEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(red_bar), 1);
    *s_abort = 0;
    prefetch_tmap(&tmap_x);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  __syncthreads();
  // The next GEMM in the stream may start its own set-up and weight streaming
  // on SMs this grid leaves; it waits (grid_dep_wait) before touching data this
  // grid writes.
  grid_dep_launch();

  // TMEM is allocated off the producer's critical path; every warp but the
  // producer needs its address (named barrier 2).
  constexpr int kTmemBarThreads = Cfg::kThreads - 32;
  uint32_t tmem_base = 0;
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), Cfg::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
    named_bar_sync(2, kTmemBarThreads);
    tc_fence_after();
    tmem_base = *s_tmem;
  } else if (warp >= 2) {
    named_bar_sync(2, kTmemBarThreads);
    tc_fence_after();
    tmem_base = *s_tmem;
  }
  const uint32_t tmem_a_base = tmem_base + (uint32_t)Cfg::kAcol0;

  if (n_local == 0) {
    // nothing to do for this CTA
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop (so addresses stay warp-uniform and live in
    // uniform registers); one elected lane issues the copies.
    // Weights are read once per token tile: stream them past L2 when there is
    // a single token tile (decode), keep them when later token tiles reuse them.
    const uint64_t pol_w = MT > 1 ? policy_evict_normal() : policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    RingPos st;
    WorkPos up;
    up.init(0, sch);
    int issued = 0;
    const uint8_t* blob = p.blob;
    int blob_mt = -1;
    // Weights do not depend on the previous kernel in the stream: the epilogue
    // warps (idle until the first accumulator) copy the first `early` stages'
    // weights before the grid dependency resolves, and the dequantisers start on
    // them as they land (own barrier). The producer only adds the activations of
    // those stages, after the wait. Each bulk copy takes ~0.3 us to issue, so
    // spreading them over four warps gets the producer to its first activation
    // load sooner.
    const int early = cmin(SL, n_local);
    const bool weights_early = (p.tile_expert == nullptr);
    grid_dep_wait();
    for (; up.j < n_local; up.next(sch)) {
      if (issued >= SL) {
        if (!mbar_wait(smem_u32(&empty_l[st.idx]), st.phase ^ 1u)) {
          if (lane == 0) atomicOr(p.err, kErrWaitProducer);
          *s_abort = 1;
          break;
        }
      }
      if (*s_abort) break;
      if (p.tile_expert != nullptr && up.mt != blob_mt) {
        blob = p.blob + (int64_t)p.tile_expert[up.mt] * p.blob_stride;
        blob_mt = up.mt;
      }
      const uint8_t* src = blob + ((int64_t)up.nt * KB + up.kb * SB) * Cfg::kPkBytes;
      uint8_t* stg = lring + st.idx * Cfg::kLStage;
      const uint32_t bar = smem_u32(&full_x[st.idx]);
      const bool weights_sent = weights_early && issued < early;
      if (elect_one()) {
        if (!weights_sent) {
          const uint32_t wbar = smem_u32(&full_w[st.idx]);
          mbar_arrive_expect_tx(wbar, Cfg::kPkStage);
          bulk_g2s(smem_u32(stg), src, Cfg::kPkStage, wbar, pol_w);
        }
        mbar_arrive_expect_tx(bar, Cfg::kXBytes);
        if (p.x3d) {
          tma_load_3d(smem_u32(stg + Cfg::kPkRegion), &tmap_x, 0, up.mt * NTOK, up.kb * Cfg::kXAtoms, bar,
                      pol_x);
        } else {
#pragma unroll
          for (int a = 0; a < Cfg::kXAtoms; ++a)
            tma_load_2d(smem_u32(stg + Cfg::kPkRegion + a * Cfg::kXAtom), &tmap_x,
                        (up.kb * Cfg::kXAtoms + a) * 64, up.mt * NTOK, bar, pol_x);
        }
      }
      __syncwarp();
      ++issued;
      st.next<SL>();
    }
    // Do not leave while copies into this CTA's shared memory are in flight:
    // wait for the completion of the last min(issued, SL) stages.
    for (int j = 0; j < cmin(issued, SL); ++j) {
      if (st.idx == 0) st.phase ^= 1u;
      st.idx = (st.idx == 0 ? SL : st.idx) - 1;
      if (!mbar_wait(smem_u32(&full_w[st.idx]), st.phase) || !mbar_wait(smem_u32(&full_x[st.idx]), st.phase)) {
        if (lane == 0) atomicOr(p.err, kErrWaitDrain);
        break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Warp-wide loop, one elected lane issues tcgen05.mma / commit.
    constexpr uint32_t idesc = make_idesc_f16(128, NTOK, IsBf16<T>::value ? 1 : 0);
    // Descriptor of stage 0; other stages and k-steps only move the start
    // address (bits 0..13, in 16-byte units), which never carries out.
    const uint64_t adesc0 = make_sw128_kmajor_desc(smem_u32(wring));
    const uint64_t bdesc0 = make_sw128_kmajor_desc(smem_u32(lring + Cfg::kPkRegion));
    RingPos sl, sd, acc;
    int seg = 0;
    bool ok = true;
    for (int u = 0; u < n_local && ok; ++seg) {
      const int seg_end = sch.seg_end(u);
      const int seg_begin = u;
      if (seg >= 2) {
        if (!mbar_wait(smem_u32(&acc_empty[acc.idx]), acc.phase ^ 1u)) {
          if (lane == 0) atomicOr(p.err, kErrWaitMma);
          *s_abort = 1;
          break;
        }
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc.idx * NTOK);
      for (; u < seg_end; ++u) {
        if (!mbar_wait(smem_u32(&full_x[sl.idx]), sl.phase) ||
            !mbar_wait(smem_u32(&full_d[sd.idx]), sd.phase)) {
          if (lane == 0) atomicOr(p.err, kErrWaitMma);
          *s_abort = 1;
          ok = false;
          break;
        }
        if (*s_abort) { ok = false; break; }
        tc_fence_after();
        const uint64_t bd = bdesc0 + (uint64_t)((sl.idx * Cfg::kLStage) >> 4);
        if (elect_one()) {
          if constexpr (Cfg::kATmem) {
            // A stage sd: kAStageCols TMEM columns, 8 per 16-wide k step
            const uint32_t at = tmem_a_base + (uint32_t)(sd.idx * Cfg::kAStageCols);
            tc_mma_f16_ts(d_tmem, at, bd, idesc, u != seg_begin ? 1u : 0u);
#pragma unroll
            for (int kk = 1; kk < 8 * SB; ++kk) {
              const uint64_t kx = (uint64_t)((kk >> 2) * (Cfg::kXAtom >> 4) + (kk & 3) * 2);
              tc_mma_f16_ts(d_tmem, at + (uint32_t)(8 * kk), bd + kx, idesc, 1u);
            }
          } else {
            const uint64_t ad = adesc0 + (uint64_t)((sd.idx * Cfg::kWStage) >> 4);
            tc_mma_f16(d_tmem, ad, bd, idesc, u != seg_begin ? 1u : 0u);
#pragma unroll
            for (int kk = 1; kk < 8 * SB; ++kk) {
              const uint64_t ka = (uint64_t)((kk >> 2) * (16384 >> 4) + (kk & 3) * 2);
              const uint64_t kx = (uint64_t)((kk >> 2) * (Cfg::kXAtom >> 4) + (kk & 3) * 2);
              tc_mma_f16(d_tmem, ad + ka, bd + kx, idesc, 1u);
            }
          }
          tc_commit(smem_u32(&empty_d[sd.idx]));
          tc_commit(smem_u32(&empty_l[sl.idx]));
        }
        __syncwarp();
        sl.next<SL>();
        sd.next<SD>();
      }
      if (ok && elect_one()) tc_commit(smem_u32(&acc_full[acc.idx]));
      __syncwarp();
      acc.next<2>();
    }
    // Every MMA issued must finish before TMEM is released.
    if (elect_one()) tc_commit(smem_u32(drain));
    __syncwarp();
    if (!mbar_wait(smem_u32(drain), 0) && lane == 0) atomicOr(p.err, kErrWaitDrain);
  } else if (warp >= Cfg::kEpiWarp0 && warp < Cfg::kEpiWarp0 + Cfg::kNumEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int f = q * 32 + lane;            // feature row within the tile
    const int etid = threadIdx.x - Cfg::kEpiWarp0 * 32;
    constexpr int kEpiThreads = Cfg::kNumEpiWarps * 32;
    if (p.tile_expert == nullptr && n_local > 0) {
      // early weight copies (see the producer); expert ids of the grouped GEMM
      // come from the previous kernel, so those wait for the producer's loop
      const uint64_t pol_w = MT > 1 ? policy_evict_normal() : policy_evict_first();
      const int early = cmin(SL, n_local);
      for (int j = warp - Cfg::kEpiWarp0; j < early; j += Cfg::kNumEpiWarps) {
        WorkPos ue;
        ue.init(j, sch);
        const uint8_t* src = p.blob + ((int64_t)ue.nt * KB + ue.kb * SB) * Cfg::kPkBytes;
        const uint32_t bar = smem_u32(&full_w[j]);
        if (elect_one()) {
          mbar_arrive_expect_tx(bar, Cfg::kPkStage);
          bulk_g2s(smem_u32(lring + j * Cfg::kLStage), src, Cfg::kPkStage, bar, pol_w);
        }
        __syncwarp();
      }
    }
    grid_dep_wait();  // outputs, workspace counters and partials belong to the previous grid until then
    if (etid == 0) *s_tpe = p.tp_world > 0 ? (uint32_t)*reinterpret_cast<volatile int*>(p.tp_epoch) : 0u;
    named_bar_sync(1, kEpiThreads);
    RingPos acc;
    for (int u = 0; u < n_local; acc.next<2>()) {
      const int tile = sch.tile_of(u);
      const int seg_end = sch.seg_end(u);
      int mt, nt;
      sch.tile_mn(tile, mt, nt);
      const int n = nt * kBlockN + f;
      int rows_here = p.M - mt * NTOK;
      if (p.rows_valid != nullptr) rows_here = cmin(rows_here, *p.rows_valid - mt * NTOK);
      rows_here = cmax(0, cmin(NTOK, rows_here));
      const int ncols = (rows_here + 15) & ~15;

      // Contributors: stream-K tiles may be cut by range boundaries; the
      // data-parallel tiles are whole.
      const bool sk = u >= sch.dp_units;
      const int r_tile = tile * KBS - sch.sk_base;  // tile start relative to the stream-K phase
      const int c_first = sk ? sch.sk_owner(r_tile) : (int)blockIdx.x;
      const int c_last = sk ? sch.sk_owner(r_tile + KBS - 1) : (int)blockIdx.x;
      const int ncontrib = c_last - c_first + 1;
      const bool split = ncontrib > 1;
      // The owner holds the tile's first unit. The tile runs past its range, so
      // this is its last segment and the other TMEM accumulator buffer is free.
      const bool owner = split && c_first == (int)blockIdx.x && p.cluster_s <= 1;
      // A split tile is the last segment of its first contributor, so each CTA
      // owns at most one: the tile's counters are indexed by that contributor.
      int32_t* const cnt = p.ws_cnt + 2 * c_first;
      const uint32_t lane_off = (uint32_t)(q * 32) << 16;
      const uint32_t t_addr = tmem_base + lane_off + (uint32_t)(acc.idx * NTOK);
      const uint32_t t_spare = tmem_base + lane_off + (uint32_t)((acc.idx ^ 1) * NTOK);
      // Partial of contributor cj (slot 0 = its first segment, 1 = its last),
      // column-major [NTOK][128]: column c of feature f at [c * 128 + f], so a
      // warp moves 128 contiguous bytes per column.
      auto part_of = [&](int cj) -> const float* {
        const int cs = (sch.sk_start(cj) >= r_tile) ? 0 : 1;
        return p.ws_part + ((int64_t)cj * 2 + cs) * (128 * NTOK);
      };

      // Scattered output (MoE): the destination rows and scales of the tile do
      // not depend on the accumulator. Each warp stages them in its own slots
      // (two dependent loads per row, all rows in flight) before waiting for it.
      int2* const rows_sm = row_slots + (warp - Cfg::kEpiWarp0) * NTOK;
      if (p.row_map != nullptr || p.row_scale != nullptr) {
        __syncwarp();  // this warp's reads of the previous tile's slots are done
        constexpr int kIt = (NTOK + 31) / 32;
        int rm[kIt];
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
          const int c = lane + 32 * i;
          int m = mt * NTOK + c;
          bool ok = c < rows_here;
          if (ok && p.row_map != nullptr) {
            m = p.row_map[m];
            ok = m < p.num_valid;  // padding rows of an expert block
          }
          rm[i] = ok ? m : -1;
        }
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
          const float sc = (rm[i] >= 0 && p.row_scale != nullptr) ? p.row_scale[rm[i]] : 1.f;
          if (lane + 32 * i < NTOK) rows_sm[lane + 32 * i] = make_int2(rm[i], __float_as_int(sc));
        }
        __syncwarp();
      }

      // Wait for the accumulator. Meanwhile an owner checks whether its peers
      // have all published. Up to 16 rows it then sums their partials (in
      // contributor order) into the spare TMEM buffer, so the fix-up costs
      // nothing once its own MMAs are done; it gives up as soon as its
      // accumulator is ready. With more rows that sum would take several round
      // trips to L2: the owner instead reduces as soon as its accumulator is
      // ready, without an arrival ticket (it knows it is the last to arrive).
      bool pre = false;
      bool published = false;
      {
        const uint32_t bar = smem_u32(&acc_full[acc.idx]);
        bool done = mbar_try_wait(bar, acc.phase);
        bool tried = false;
        const uint64_t t0 = done ? 0 : globaltimer_ns();
        while (!done) {
          if (owner && !tried) {
            // every lane acquires for itself; the decision is warp-uniform
            if (__all_sync(0xffffffffu, ld_acquire_gpu(&cnt[1]) == ncontrib - 1)) {
              tried = true;
              published = true;
              bool complete = rows_here <= 16;
#pragma unroll 1
              for (int c0 = 0; complete && c0 < rows_here; c0 += 8) {
                if (c0 > 0 && mbar_test_wait(bar, acc.phase)) {
                  complete = false;
                  done = true;
                  break;
                }
                float sum[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) sum[i] = 0.f;
#pragma unroll 1
                for (int cj = c_first + 1; cj <= c_last; ++cj) {
                  const float* src = part_of(cj) + c0 * 128 + f;
                  float a[8];
#pragma unroll
                  for (int i = 0; i < 8; ++i) a[i] = (c0 + i < rows_here) ? __ldcg(src + i * 128) : 0.f;
#pragma unroll
                  for (int i = 0; i < 8; ++i) sum[i] += a[i];
                }
                uint32_t sv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) sv[i] = __float_as_uint(sum[i]);
                tmem_st8(t_spare + (uint32_t)c0, sv);
              }
              tmem_st_wait();
              pre = complete && rows_here <= 16;
              if (done) break;
            }
          }
          done = mbar_try_wait_hint(bar, acc.phase, (owner && !tried) ? 1000u : 20000u);
          if (!done && globaltimer_ns() - t0 > AWQB_WAIT_TIMEOUT_NS) break;
        }
        if (!done) {
          atomicOr(p.err, kErrWaitEpilogue);
          *s_abort = 1;
          break;
        }
        if (owner && !tried && rows_here > 16)
          published = __all_sync(0xffffffffu, ld_acquire_gpu(&cnt[1]) == ncontrib - 1);
      }
      tc_fence_after();

      float bias_v = 0.f;
      if (p.bias != nullptr && n < p.N) bias_v = (float)reinterpret_cast<const T*>(p.bias)[n];
      // Stores rows c0 .. c0+cnt-1 of this thread's feature. The output row of
      // each (row_map) and its scale (row_scale) are read once per chunk by
      // lanes 0..15 and broadcast with shuffles (warp-uniform loop).
      auto store_row_vals = [&](int c0, const float* vals, int cnt) {
        if (p.silu_mul) {
          // Column 2j is gate j, column 2j + 1 is up j: the pair sits in
          // neighbouring lanes. One shuffle swaps them; the gate lane writes the
          // even token columns, the up lane the odd ones.
          const int odd = f & 1;
          const int no = n >> 1;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c >= cnt) break;
            const float mine = vals[c] + bias_v;
            const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
            if ((c & 1) == odd && c0 + c < rows_here && n < p.N) {
              const float g = odd ? other : mine;
              const float u = odd ? mine : other;
              reinterpret_cast<T*>(p.y)[(int64_t)(mt * NTOK + c0 + c) * p.ldy + no] = (T)(silu_fast(g) * u);
            }
          }
          return;
        }
        if (p.tp_world > 0) {  // fused all-reduce: tagged words to every rank's landing slot (no bias yet)
          if (n >= p.N) return;
          const uint32_t e = *s_tpe;
          const int64_t base = (int64_t)(e & 1u) * p.tp_half +
                               ((int64_t)p.tp_rank * p.tp_rows + mt * NTOK + c0) * p.N + n;
          const int lim = cmin(cnt, rows_here - c0);
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c < lim) tp_put(p.tp_land, p.tp_world, base + (int64_t)c * p.N, vals[c], e + 1u);
          return;
        }
        if (p.row_map == nullptr && p.row_scale == nullptr) {  // dense GEMM: rows in order
          if (n >= p.N) return;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c >= cnt || c0 + c >= rows_here) break;
            reinterpret_cast<T*>(p.y)[(int64_t)(mt * NTOK + c0 + c) * p.ldy + n] = (T)(vals[c] + bias_v);
          }
          return;
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          if (c >= cnt) break;
          const int2 rs = rows_sm[c0 + c];  // same address in every lane: broadcast
          if (rs.x >= 0 && n < p.N) {
            float val = vals[c] + bias_v;
            if (p.row_scale != nullptr) val *= __int_as_float(rs.y);
            reinterpret_cast<T*>(p.y)[(int64_t)rs.x * p.ldy + n] = (T)val;
          }
        }
      };
      // Fused all-reduce, after this thread has written its final values of the
      // tile to every rank: wait for each rank's word of each of its values
      // (tag of this call), sum them in rank order, add the bias, store.
      // (The reduce-scatter mode is only used with cluster split-K plans; the
      // stream-K path always exchanges all-to-all.)
      auto tp_finish = [&]() {
        if (n >= p.N) return;
        const uint32_t e = *s_tpe;
        const float bv = p.bias != nullptr ? (float)reinterpret_cast<const T*>(p.bias)[n] : 0.f;
        tp_finalize_column<T>(p.tp_land[p.tp_rank] + (int64_t)(e & 1u) * p.tp_half + (int64_t)mt * NTOK * p.N + n,
                              reinterpret_cast<T*>(p.y) + (int64_t)mt * NTOK * p.ldy + n, p.ldy, p.N, p.tp_rows,
                              p.tp_world, rows_here, bv, e + 1u, p.err);
      };

      if (split && p.cluster_s > 1) {
        // Cluster split-K: this tile is the CTA's only segment, so the load ring
        // is idle. The partial goes to shared memory as [row][128 features]; the
        // cluster reduces it after the final barrier (kernel end).
        float* sp = reinterpret_cast<float*>(lring) + f;
#pragma unroll 1
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(t_addr + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c0 + c < rows_here) sp[(c0 + c) * 128] = __uint_as_float(v[c]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc.idx]));
        u = seg_end;
        continue;
      }
      const bool fast = split && named_bar_and(1, kEpiThreads, owner && pre);
      // An owner whose peers have all published reduces at once (no ticket).
      const bool fetch = split && !fast && named_bar_and(1, kEpiThreads, owner && published);
      if (!split || fast) {
        // Whole tile, or an owner with its peers' sum ready: final values now.
#pragma unroll 1
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          uint32_t v[16];
          float vals[16];
          tmem_ld16(t_addr + c0, v);
          if (fast) {
            uint32_t w[16];
            tmem_ld16(t_spare + c0, w);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 16; ++c) vals[c] = __uint_as_float(w[c]) + __uint_as_float(v[c]);
          } else {
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 16; ++c) vals[c] = __uint_as_float(v[c]);
          }
          store_row_vals(c0, vals, 16);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc.idx]));
        if (fast && etid == 0) {  // every peer has published; nobody else touches the counters
          cnt[0] = 0;
          cnt[1] = 0;
        }
        if (p.tp_world > 0) tp_finish();
      } else {
        // Take an arrival ticket. The last contributor to arrive reduces the
        // tile: it keeps its own partial in TMEM and waits for the others to
        // publish theirs. Everyone else publishes. A reducer only ever waits for
        // CTAs that have already arrived (so are running): no co-residency of
        // the grid is assumed.
        if (etid == 0) {
          if (fetch) {
            s_flag[acc.idx] = 1;
          } else {
            const int prev = atom_add_relaxed_gpu(&cnt[0], 1);
            s_flag[acc.idx] = (prev == ncontrib - 1) ? 1 : 0;
          }
        }
        named_bar_sync(1, kEpiThreads);
        const bool reducer = s_flag[acc.idx] != 0;
        if (!reducer) {
          // Publish: slot 0 holds this CTA's first segment, slot 1 its last.
          const int slot = (u == sch.dp_units) ? 0 : 1;  // first stream-K segment?
          float* part = p.ws_part + ((int64_t)blockIdx.x * 2 + slot) * (128 * NTOK) + f;
#pragma unroll 1
          for (int c0 = 0; c0 < ncols; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(t_addr + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 16; ++c)
              if (c0 + c < rows_here) __stcg(part + (c0 + c) * 128, __uint_as_float(v[c]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc.idx]));
          // The block barrier orders every thread's partial stores before thread
          // 0's release-ordered add (cumulativity).
          named_bar_sync(1, kEpiThreads);
          if (etid == 0) red_add_release_gpu(&cnt[1], 1);
        } else {
          // Sequence order of the sum: c_first+1 .. c_last, then c_first. On the
          // CTA's last segment the load ring is idle (every MMA has completed), so
          // the peers' partials come in with one bulk copy each; otherwise they
          // are loaded into registers.
          const int me = (int)blockIdx.x;
          const int s_me = (me == c_first) ? ncontrib - 1 : me - c_first - 1;
          const int peer_bytes = rows_here * 128 * 4;
          const bool bulk = seg_end == n_local && (int64_t)(ncontrib - 1) * peer_bytes <= (int64_t)SL * Cfg::kLStage;
          if (etid == 0) {
            // Bounded wait for the other ncontrib - 1 partials.
            int ok = 1;
            if (!fetch && ld_acquire_gpu(&cnt[1]) != ncontrib - 1) {
              const uint64_t t0 = globaltimer_ns();
              while (ld_acquire_gpu(&cnt[1]) != ncontrib - 1) {
                if (globaltimer_ns() - t0 > AWQB_WAIT_TIMEOUT_NS) {
                  atomicOr(p.err, kErrWaitEpilogue);
                  ok = 0;
                  break;
                }
              }
            }
            if (ok) {
              cnt[0] = 0;
              cnt[1] = 0;
              if (bulk && peer_bytes > 0) {
                fence_proxy_async_global();  // peers' generic stores -> bulk-copy reads
                const uint32_t rb = smem_u32(red_bar);
                mbar_arrive_expect_tx(rb, (uint32_t)((ncontrib - 1) * peer_bytes));
                for (int s = 0; s < ncontrib; ++s) {
                  if (s == s_me) continue;
                  const int cj = (s < ncontrib - 1) ? c_first + 1 + s : c_first;
                  const int slot = s < s_me ? s : s - 1;
                  bulk_g2s(smem_u32(lring + (size_t)slot * peer_bytes), part_of(cj), (uint32_t)peer_bytes, rb,
                           policy_evict_first());
                }
              }
            }
            s_flag[acc.idx] = ok ? 1 : 2;
          }
          named_bar_sync(1, kEpiThreads);
          if (s_flag[acc.idx] == 1) {
            bool have = true;
            if (bulk && peer_bytes > 0) {
              have = mbar_wait(smem_u32(red_bar), 0);
              if (!have && etid == 0) atomicOr(p.err, kErrWaitEpilogue);
            }
            const float* sm = reinterpret_cast<const float*>(lring) + f;
#pragma unroll 1
            for (int c0 = 0; have && c0 < rows_here; c0 += 8) {
              uint32_t ov[8];
              tmem_ld8(t_addr + c0, ov);
              tmem_ld_wait();
              float sum[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) sum[i] = 0.f;
#pragma unroll 1
              for (int s = 0; s < ncontrib; ++s) {
                float a[8];
                if (s == s_me) {
#pragma unroll
                  for (int i = 0; i < 8; ++i) a[i] = __uint_as_float(ov[i]);
                } else if (bulk) {
                  const float* src = sm + (size_t)(s < s_me ? s : s - 1) * (peer_bytes / 4) + c0 * 128;
#pragma unroll
                  for (int i = 0; i < 8; ++i) a[i] = (c0 + i < rows_here) ? src[i * 128] : 0.f;
                } else {
                  const int cj = (s < ncontrib - 1) ? c_first + 1 + s : c_first;
                  const float* src = part_of(cj) + c0 * 128 + f;
#pragma unroll
                  for (int i = 0; i < 8; ++i) a[i] = (c0 + i < rows_here) ? __ldcg(src + i * 128) : 0.f;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) sum[i] += a[i];
              }
              store_row_vals(c0, sum, 8);
            }
            if (p.tp_world > 0) tp_finish();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc.idx]));
        }
      }
      u = seg_end;
    }
    tc_fence_before();
  } else if (warp >= Cfg::kDqWarp0) {
    // ------------------------------------------------------------ dequantisers
    // Group g of 8 warps takes stages g, g+2, ...: two stages are dequantised
    // at once, so one group's load / TMEM-store / barrier latencies overlap the
    // other group's arithmetic. Warp w writes TMEM lanes 32*(w%4).. (the
    // hardware restriction), so a thread owns weight row r = 32*(w%4) + lane and,
    // in every block of its stage, the eight words (64 k) of half h: two 16-byte
    // shared loads and eight dequantised 16-byte chunks per block.
    const int wi = warp - Cfg::kDqWarp0;      // 0..15
    const int dg = wi >> 3;                   // group 0 / 1
    const int h = (wi >> 2) & 1;              // 64-wide half of each block
    const int q = warp & 3;                   // TMEM lane quarter
    const int r = q * 32 + lane;
    const int rsw = r & 7;
    const uint32_t ld_off = (uint32_t)((2 * h * 128 + r) << 4);
    const uint32_t st_off = (uint32_t)(h * 16384 + r * 128);
    int il = dg % SL, pl = (dg >= SL);    // load-ring slot / phase of this group's current stage
    int id = dg % SD, pd = (dg >= SD);    // A-ring slot / phase
    for (int u = dg; u < n_local; u += 2) {
      if (!mbar_wait(smem_u32(&full_w[il]), (uint32_t)pl)) {
        atomicOr(p.err, kErrWaitDequant);
        *s_abort = 1;
        break;
      }
      if (u >= SD) {
        if (!mbar_wait(smem_u32(&empty_d[id]), (uint32_t)pd ^ 1u)) {
          atomicOr(p.err, kErrWaitDequant);
          *s_abort = 1;
          break;
        }
      }
      if (*s_abort) break;
      if constexpr (Cfg::kATmem) tc_fence_after();  // order our TMEM stores after the MMAs that read the slot
      const uint8_t* pk = lring + il * Cfg::kLStage;
#pragma unroll
      for (int blk = 0; blk < SB; ++blk) {
        const uint8_t* pkb = pk + blk * Cfg::kPkBytes;
        typename DQ::Terms terms[GPB >= 4 ? 2 : 1];
        {
          uint16_t sb;
          uint32_t z;
          if constexpr (GPB >= 4) {
            block_scale_zero(pkb, GPB, 2 * h, r, sb, z);
            terms[0] = DQ::make(sb, z);
            block_scale_zero(pkb, GPB, 2 * h + 1, r, sb, z);
            terms[1] = DQ::make(sb, z);
          } else {
            block_scale_zero(pkb, GPB, GPB == 2 ? h : 0, r, sb, z);
            terms[0] = DQ::make(sb, z);
          }
        }
        const uint4 v0 = *reinterpret_cast<const uint4*>(pkb + ld_off);
        const uint4 v1 = *reinterpret_cast<const uint4*>(pkb + ld_off + 128 * 16);
        const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        if constexpr (Cfg::kATmem) {
          uint32_t o[32];
#pragma unroll
          for (int jl = 0; jl < 8; ++jl) {
            const uint4 t = DQ::dq8(wv[jl], terms[GPB >= 4 ? (jl >> 2) : 0]);
            o[4 * jl] = t.x;
            o[4 * jl + 1] = t.y;
            o[4 * jl + 2] = t.z;
            o[4 * jl + 3] = t.w;
          }
          tmem_st32(tmem_a_base + ((uint32_t)(q * 32) << 16) +
                        (uint32_t)(id * Cfg::kAStageCols + blk * 64 + h * 32),
                    o);
        } else {
          uint8_t* wt = wring + id * Cfg::kWStage + st_off;
#pragma unroll
          for (int jl = 0; jl < 8; ++jl) {
            const uint4 o = DQ::dq8(wv[jl], terms[GPB >= 4 ? (jl >> 2) : 0]);
            *reinterpret_cast<uint4*>(wt + ((jl ^ rsw) << 4)) = o;
          }
        }
      }
      if constexpr (Cfg::kATmem) {
        tmem_st_wait();
        tc_fence_before();
      } else {
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&full_d[id]));
        mbar_arrive(smem_u32(&empty_l[il]));
      }
      il += 2; if (il >= SL) { il -= SL; pl ^= 1; }
      id += 2; if (id >= SD) { id -= SD; pd ^= 1; }
    }
  }

  __syncwarp();  // roles end after per-lane waits: reconverge before the aligned barrier
  __syncthreads();
  if (p.cluster_s > 1) {
    // Cluster split-K finale: every CTA of the cluster holds a partial of the
    // same tile in shared memory ([row][128 features] fp32). Rank r sums the
    // features of its slice, whole 16-byte quads [4 (32 r / S), 4 (32 (r+1) / S)),
    // over the S partials in rank order (deterministic), reading its peers'
    // shared memory directly (one 16-byte load per peer and quad), and stores
    // them. It then signals that it is done reading its peers; the final wait
    // keeps its own shared memory alive until they are done reading it.
    cluster_sync_all();
    const int S = p.cluster_s;
    const int rank = (int)cluster_ctarank();
    const int tile = sch.tile_of(0);
    int mt, nt;
    sch.tile_mn(tile, mt, nt);
    const int rows_here = n_local > 0 ? cmax(0, cmin(NTOK, p.M - mt * NTOK)) : 0;
    const int f0 = 4 * (rank * 32 / S);
    const int nf = 4 * ((rank + 1) * 32 / S) - f0;
    const int nq = nf >> 2;
    const uint32_t tp_epoch = p.tp_world > 0 ? (uint32_t)*reinterpret_cast<volatile int*>(p.tp_epoch) : 0u;
    const int tp_par = (int)(tp_epoch & 1u);
    const uint32_t tp_tag = tp_epoch + 1u;
    const uint32_t base_sm = smem_u32(lring);
    // Fused all-reduce: one feature per thread, so that the thread that sends a
    // value is the one that later waits for that value's words (its own rank's
    // word is then its own store: no extra round trip to see it).
    for (int e = threadIdx.x; p.tp_world > 0 && e < nf * rows_here; e += Cfg::kThreads) {
      const int c = e / nf;
      const int f = f0 + (e - c * nf);
      const int n = nt * kBlockN + f;
      if (n >= p.N) continue;
      const uint32_t off = base_sm + (uint32_t)((c * 128 + f) * 4);
      float v = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < S) v += ld_dsmem_f32(mapa_shared(off, (uint32_t)r));
      const int m = mt * NTOK + c;
      const int64_t o = (int64_t)tp_par * p.tp_half + ((int64_t)p.tp_rank * p.tp_rows + m) * p.N + n;
      if (p.tp_rsag)
        st_tagged_sys(p.tp_land[nt % p.tp_world] + o, v, tp_tag);
      else
        for (int d = 0; d < p.tp_world; ++d) st_tagged_sys(p.tp_land[d] + o, v, tp_tag);
    }
    // Dense output in one 8-byte store per quad when the rows are 8-byte aligned.
    const bool vec_out = (p.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(p.y) & 7) == 0;
    for (int e = threadIdx.x; p.tp_world == 0 && e < nq * rows_here; e += Cfg::kThreads) {
      const int c = e / nq;
      const int f = f0 + 4 * (e - c * nq);
      const int n0 = nt * kBlockN + f;
      if (n0 >= p.N) continue;  // past the last feature: nothing to load or store
      const uint32_t off = base_sm + (uint32_t)((c * 128 + f) * 4);
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r < S) {
          const float4 a = ld_dsmem_v4(mapa_shared(off, (uint32_t)r));
          v[0] += a.x;
          v[1] += a.y;
          v[2] += a.z;
          v[3] += a.w;
        }
      }
      const int m = mt * NTOK + c;
      if (vec_out && n0 + 3 < p.N) {
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float out = v[j];
          if (p.bias != nullptr) out += (float)reinterpret_cast<const T*>(p.bias)[n0 + j];
          const T t = (T)out;
          h[j] = *reinterpret_cast<const uint16_t*>(&t);
        }
        *reinterpret_cast<uint2*>(reinterpret_cast<T*>(p.y) + (int64_t)m * p.ldy + n0) =
            make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
        continue;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + j;
        if (n >= p.N) break;
        float out = v[j];
        if (p.bias != nullptr) out += (float)reinterpret_cast<const T*>(p.bias)[n];
        reinterpret_cast<T*>(p.y)[(int64_t)m * p.ldy + n] = (T)out;
      }
    }
    // Every value loaded from a peer above has been consumed by a store, so
    // the loads are complete: a relaxed arrive is enough to tell the peers that
    // their shared memory is no longer read (no need to wait for the global
    // stores to be acknowledged).
    cluster_arrive_relaxed();
    if (p.tp_world > 0) tp_cluster_finish<T>(p, nt * kBlockN + f0, nf, mt * NTOK, rows_here, tp_epoch);
    cluster_wait();
  }
  if (p.tp_world > 0 && threadIdx.x == 0) {
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
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace awqb
