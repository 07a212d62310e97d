// Host side of the W4A16 GEMM: argument checks, tile-size choice, TMA tensor
// map for the activations, launch, and the C-ABI entry points declared in
// include/awqb200.h.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <atomic>
#include <mutex>

#include "awqb200.h"
#include "awqb_common.h"
#include "awqb_gemm.cuh"
#include "awqb_gemv.cuh"

namespace awqb {

__device__ uint32_t g_awqb_err;  // OR of DeviceError bits, cleared by awqb_clear_device_error

namespace {

constexpr int kMaxDevices = 64;

uint32_t* device_err_ptr() {
  static uint32_t* ptrs[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_awqb_err) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<uint32_t*>(p);
  }
  return ptrs[dev];
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Activation tensor map, 128-byte swizzle, out-of-range elements read as zero.
// K % 64 == 0: a 3-D view {64, rows, K/64} (strides K*2 and 128 bytes) whose box
// {64, ntok, atoms} brings a whole stage (atoms x 64 k) in one load; otherwise
// a 2-D view with box {64, ntok} and one load per 64-wide atom. *is3d reports
// which.
int make_x_tensor_map(CUtensorMap* tm, const void* x, int64_t rows, int64_t K, int ntok, int atoms, int* is3d) {
  auto enc = tensor_map_encoder();
  AWQB_REQUIRE(enc != nullptr, kCudaError, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint32_t estride[3] = {1u, 1u, 1u};
  CUresult r;
  if (K % 64 == 0) {
    cuuint64_t gdim[3] = {64, (cuuint64_t)rows, (cuuint64_t)(K / 64)};
    cuuint64_t gstride[2] = {(cuuint64_t)K * 2, 128};
    cuuint32_t box[3] = {64u, (cuuint32_t)ntok, (cuuint32_t)atoms};
    r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(x), gdim, gstride, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    *is3d = 1;
  } else {
    cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64u, (cuuint32_t)ntok};
    r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(x), gdim, gstride, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    *is3d = 0;
  }
  AWQB_REQUIRE(r == CUDA_SUCCESS, kCudaError, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return kOk;
}

// Token tile: the smallest built tile that holds a decode batch; 128 (weights
// in TMEM, 256-k stages) up to a few thousand tokens, where it keeps more tiles
// in flight than SMs; 256 (weights in shared memory, each dequantised weight
// reused by twice as many tokens) for the largest prefill batches.
// Measured on B200 over the Llama-3 / Qwen3 projection shapes: 64-token tiles
// win up to about M = 1024, 128-token tiles (five 128-k load stages) above;
// the 256-token tile (operand A in shared memory, two load stages) never wins
// and is only built for explicit requests.
// Token tile by M, swept on B200 over the decode and Qwen3-4B prefill shapes
// (128-token tiles are as fast or faster for every shape from M = 1024 on).
int choose_ntok(int64_t M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 512) return 64;
  return 128;
}

// Token tiles per raster group. Weights that fit comfortably in the 126 MB L2
// are re-read from L2 by every token tile, and walking all feature tiles of
// one token tile first maximises activation sharing; larger weights (and MoE
// experts, whose token tiles differ in expert) are shared by groups of 8 token
// tiles so that each weight tile is read from DRAM about once per group.
int raster_group_m(int64_t K, int64_t N, bool grouped) {
  const int64_t weight_bytes = K * N / 2;
  return (grouped || weight_bytes > (40ll << 20)) ? 8 : 1;
}

// 128-k blocks per pipeline stage of the kernel built for this token tile.
int stage_blocks(int ntok) { return ntok <= 64 ? 2 : 1; }  // must match GemmCfg::kSB

struct Plan {
  int ntok, gpb;
  int NT, KB, MT;
  int64_t ctas;
  int64_t cnt_bytes, part_bytes;
  int cluster_s;  // >= 2: cluster split-K launch (one tile per cluster of cluster_s CTAs)
};

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// At most kMaxCtas persistent CTAs; two int32 counters each.
constexpr int kMaxCtas = 1024;
constexpr int64_t kCounterBytes = 2 * 4 * kMaxCtas;

bool valid_group(int64_t G) { return G == 32 || G == 64 || (G >= 128 && G % 128 == 0); }

// How many clusters of S GEMM CTAs (one CTA per SM) the device runs at once;
// cached per device. Every instantiation of the kernel needs nearly all of an
// SM's shared memory, so one representative answers for all of them.
int max_active_clusters(int S) {
  static std::atomic<int> cache[kMaxDevices][9];
  static std::once_flag init_flag;
  std::call_once(init_flag, [] {
    for (auto& row : cache)
      for (auto& v : row) v.store(-1);
  });
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || S < 1 || S > 8) return 0;
  int v = cache[dev][S].load();
  if (v >= 0) return v;
  using Cfg = GemmCfg<16, 1>;
  auto kern = awq_gemm_kernel<__nv_bfloat16, 16, 1>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(S * 64));
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[dev][S].store(n);
  return n;
}

// allow_cluster: a dense GEMM whose tiles fill at most half the SMs runs as
// cluster split-K (each tile's stages split over a cluster of S CTAs whose
// partials are reduced through distributed shared memory) when all T clusters
// fit on the device at once.
// prefer_cluster: take cluster split-K whenever it fits (the fused all-reduce,
// whose per-value exchange is cheapest with the cluster's all-thread finale).
int make_plan(int64_t M, int64_t K, int64_t N, int64_t G, int ntok, int64_t ctas, Plan* pl,
              bool allow_cluster = false, bool prefer_cluster = false) {
  AWQB_REQUIRE(M >= 0 && K > 0 && N > 0, kInvalidArgument, "bad GEMM sizes M=%lld K=%lld N=%lld",
               (long long)M, (long long)K, (long long)N);
  AWQB_REQUIRE(valid_group(G), kUnsupported, "group size %lld not supported (32, 64 or a multiple of 128)",
               (long long)G);
  AWQB_REQUIRE(K % G == 0, kInvalidArgument, "K=%lld is not a multiple of the group size %lld",
               (long long)K, (long long)G);
  AWQB_REQUIRE(N % 8 == 0, kInvalidArgument, "N=%lld is not a multiple of 8", (long long)N);
  AWQB_REQUIRE(M < (1ll << 31) && K < (1ll << 31) && N < (1ll << 31), kUnsupported, "sizes too large");
  AWQB_REQUIRE((M / 16 + 1) * ((N + 127) / 128) * ((K + 127) / 128) < (1ll << 31), kUnsupported,
               "problem has too many work units");
  pl->ntok = ntok > 0 ? ntok : choose_ntok(M);
  AWQB_REQUIRE(pl->ntok == 16 || pl->ntok == 32 || pl->ntok == 64 || pl->ntok == 128 ||
                   pl->ntok == 256,
               kInvalidArgument, "token tile %d not built", pl->ntok);
  pl->gpb = groups_per_block((int)G);
  pl->NT = (int)(round_up(N, kBlockN) / kBlockN);
  pl->KB = (int)blob_kblocks(K);
  pl->MT = (int)((M + pl->ntok - 1) / pl->ntok);
  const int64_t U = (int64_t)pl->MT * pl->NT * (pl->KB / stage_blocks(pl->ntok));
  int64_t c = ctas > 0 ? ctas : device_sm_count();
  pl->cluster_s = 1;
  if (ctas <= 0 && allow_cluster) {
    const int64_t tiles = (int64_t)pl->MT * pl->NT;
    const int64_t kbs = pl->KB / stage_blocks(pl->ntok);
    if (tiles >= 1 && 2 * tiles <= c) {
      int64_t S = std::min<int64_t>(std::min<int64_t>(8, c / tiles), kbs);
      while (S >= 2 && max_active_clusters((int)S) < tiles) --S;
      if (S >= 2) {
        // Cluster split-K saves the global reduction (more the more rows it
        // reduces and the more contributors stream-K would give each tile) but
        // streams on tiles * S CTAs instead of all of them. Extra stages a CTA
        // streams, in hundredths, against a threshold measured on B200 over the
        // Llama-3 8B / 70B (TP 1..8) decode shapes (one stage ~0.48 us).
        const int64_t extra = ((kbs + S - 1) / S) * 100 - tiles * kbs * 100 / c;
        const int64_t rows = std::min<int64_t>(M, pl->ntok);
        const int64_t limit = rows <= 8 ? 115 : rows <= 16 ? 210 : rows <= 32 ? 310 : 420;
        if (extra <= limit || tiles <= 20 || prefer_cluster) pl->cluster_s = (int)S;
      }
    }
    if (pl->cluster_s > 1) c = tiles * pl->cluster_s;
  }
  if (ctas <= 0 && pl->cluster_s == 1) {
    // Larger token tiles make each split tile's partials bigger to reduce:
    // cap the contributors per tile.
    const int64_t tiles = (int64_t)pl->MT * pl->NT;
    const int64_t max_contrib = pl->ntok <= 16 ? 1 << 20 : pl->ntok <= 32 ? 6 : pl->ntok <= 64 ? 4 : 2;
    if (c > tiles * max_contrib) c = tiles * max_contrib;
  }
  if (c > U) c = U;
  if (c < 1) c = 1;
  pl->ctas = c;
  AWQB_REQUIRE(c <= kMaxCtas, kInvalidArgument, "ctas=%lld above the limit %d", (long long)c, kMaxCtas);
  // The kernel's stream-K arithmetic is 32-bit: its unit indices times the CTA
  // count stay below 2 C^2 (stages per tile).
  AWQB_REQUIRE(2 * c * c * (pl->KB / stage_blocks(pl->ntok)) < (1ll << 31), kUnsupported,
               "K=%lld too large for %lld CTAs", (long long)K, (long long)c);
  // Counters live in a fixed region at the start of every workspace, so calls
  // with different plans sharing one workspace never write partials over them.
  pl->cnt_bytes = kCounterBytes;
  // Cluster split-K reduces through shared memory: no partials in the workspace.
  pl->part_bytes = pl->cluster_s > 1 ? 0 : c * 2 * 128 * (int64_t)pl->ntok * 4;
  // Narrow outputs at mid M: 64-token tiles can be too many for cluster split-K
  // while 128-token tiles are not (e.g. N = 2560, M = 256: 80 tiles vs 40;
  // measured 21.3 us stream-K vs 13.9 us cluster on B200). Take the cluster plan.
  if (ntok == 0 && ctas <= 0 && allow_cluster && pl->cluster_s == 1 && pl->ntok == 64 && M > 64) {
    Plan p2;
    if (make_plan(M, K, N, G, 128, 0, &p2, allow_cluster, prefer_cluster) == kOk && p2.cluster_s > 1) *pl = p2;
  }
  return kOk;
}

// pdl: launch as a programmatic dependent of the previous kernel in the stream
// (the kernel waits for it before touching any data it may have written).
// Not used for the grouped path, whose row count comes from the previous kernel
// and is read at kernel start.
template <typename T, int NTOK, int GPB>
int launch_t(const CUtensorMap& tm, const GemmParams& p, int64_t ctas, bool pdl, cudaStream_t stream) {
  AWQB_REQUIRE(p.cluster_s <= 1 || ctas % p.cluster_s == 0, kInvalidArgument, "grid not a multiple of the cluster");
  using Cfg = GemmCfg<NTOK, GPB>;
  auto kern = awq_gemm_kernel<T, NTOK, GPB>;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  AWQB_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    AWQB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.cluster_s > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)p.cluster_s;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  AWQB_CUDA(cudaLaunchKernelEx(&cfg, kern, tm, p));
  return kOk;
}

template <typename T, int NTOK>
int launch_g(const CUtensorMap& tm, const GemmParams& p, int gpb, int64_t ctas, bool pdl, cudaStream_t s) {
  switch (gpb) {
    case 1: return launch_t<T, NTOK, 1>(tm, p, ctas, pdl, s);
    case 2: return launch_t<T, NTOK, 2>(tm, p, ctas, pdl, s);
    case 4: return launch_t<T, NTOK, 4>(tm, p, ctas, pdl, s);
  }
  AWQB_REQUIRE(false, kUnsupported, "groups per block %d not built", gpb);
  return kUnsupported;
}

template <typename T>
int launch_n(const CUtensorMap& tm, const GemmParams& p, const Plan& pl, bool pdl, cudaStream_t s) {
  switch (pl.ntok) {
    case 16: return launch_g<T, 16>(tm, p, pl.gpb, pl.ctas, pdl, s);
    case 32: return launch_g<T, 32>(tm, p, pl.gpb, pl.ctas, pdl, s);
    case 64: return launch_g<T, 64>(tm, p, pl.gpb, pl.ctas, pdl, s);
    case 128: return launch_g<T, 128>(tm, p, pl.gpb, pl.ctas, pdl, s);
    case 256: return launch_g<T, 256>(tm, p, pl.gpb, pl.ctas, pdl, s);
  }
  AWQB_REQUIRE(false, kUnsupported, "token tile %d not built", pl.ntok);
  return kUnsupported;
}

// Peer-memory exchange of one tensor-parallel group, as seen by one rank: one
// device allocation per rank holds [2 parities][world][rows][max_n] landing
// words (8 bytes: fp32 value + call tag) and a call counter pair; every rank
// maps every peer's allocation (CUDA IPC).
struct TpExchange {
  int rank = 0, world = 1, device = 0;
  int64_t rows = 0, max_n = 0;
  int64_t half_words = 0;    // landing words per parity
  int64_t final_half = 0;    // final words (reduce-scatter mode) per parity
  int mode = 0;              // 0 auto, 1 all-to-all, 2 reduce-scatter + all-gather
  void* local = nullptr;     // this rank's allocation
  void* base[8] = {};        // every rank's allocation as mapped here
  bool opened = false;
  int64_t land_bytes() const { return 2 * half_words * 8; }
  int64_t final_bytes() const { return 2 * final_half * 4; }
  int64_t total_bytes() const { return land_bytes() + final_bytes() + 256; }
  uint2* land(int r) const { return static_cast<uint2*>(base[r]); }
  uint32_t* final_words(int r) const {
    return reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(base[r]) + land_bytes());
  }
  int32_t* epoch() const {
    return reinterpret_cast<int32_t*>(static_cast<uint8_t*>(local) + land_bytes() + final_bytes());
  }
};

// ---------------------------------------------------------------------------
// Small-batch path (awqb_gemv.cuh): M <= kGemvMaxM, no workspace.
constexpr int kGemvMaxM = 32;

// Whether awqb_gemm takes the small-batch kernel (measured against the
// tcgen05 kernel on B200 over the Llama-3-8B decode projections, whole and
// sharded 8 ways): up to 8 rows always; up to 16 rows unless the output is
// wide (N >= 16384: gate_up at M = 16, 21.3 vs 26.5 us; down at M = 16 is
// 13.2 vs 14.2 us); up to 32 rows for problems of at most 16 Mi weights
// (O 4096 x 4096 at M = 32: 8.0 vs 8.7 us). Above, the tcgen05 kernel's
// larger MMAs win.
bool gemv_takes(int64_t M, int64_t K, int64_t N) {
  if (M < 1 || M > kGemvMaxM) return false;
  if (M <= 8) return true;
  if (M <= 16) return N < 16384;
  return K * N <= (16ll << 20);
}

struct GemvPlan {
  int F = 0, MT = 0, W = 0, ring = 0, stages = 0, kb_real = 0, gpb = 1;
  int64_t ctas = 0;
  int64_t smem = 0;
};

template <int F, int MT, int GPB, int W>
int64_t gemv_stage_bytes(int M) { return GemvCfg<F, MT, GPB, W>::stage_bytes(M); }

// Stage size of a built configuration (0 if not built). It does not depend on
// MT.
int64_t gemv_stage_bytes_rt(int F, int W, int gpb, int M) {
  switch ((F * 32 + W) * 8 + gpb) {
#define AWQB_SB(f, w, g) \
  case ((f) * 32 + (w)) * 8 + (g): return gemv_stage_bytes<f, 8, g, w>(M);
    AWQB_SB(16, 16, 1) AWQB_SB(16, 16, 2) AWQB_SB(16, 16, 4)
    AWQB_SB(32, 16, 1) AWQB_SB(32, 16, 2) AWQB_SB(32, 16, 4)
    AWQB_SB(32, 8, 1) AWQB_SB(32, 8, 2) AWQB_SB(32, 8, 4)
    AWQB_SB(64, 8, 1) AWQB_SB(64, 8, 2) AWQB_SB(64, 8, 4)
#undef AWQB_SB
  }
  return 0;
}

bool gemv_built(int F, int W) { return (W == 16 && (F == 16 || F == 32)) || (W == 8 && (F == 32 || F == 64)); }

// Shared memory one SM gives a GEMV launch's CTAs when several share it (about
// half of the SM, so that the next kernel's CTAs can start beside them and
// prefetch their weights under programmatic dependent launch); a launch with
// one CTA per SM may use more.
constexpr int64_t kGemvSmemPerSm = 110 * 1024;
constexpr int64_t kGemvSmemAlone = 160 * 1024;
constexpr int64_t kGemvSmemFixed = 1024 + 256;  // alignment slack + barriers

// Configuration, from sweeps on B200 over the Llama-3-8B decode projections
// (M = 1..16, every built slice / warp count / ring depth). What matters most
// is that the CTAs fit on the SMs in one wave: a 16-warp CTA with 32-feature
// slices takes one SM, an 8-warp CTA a third of one.
//  * more than 8 rows: 8 warps, 64-feature slices from 6144 outputs (the
//    activation tile is read once per 64 features), 32 below;
//  * outputs of at least 16384 features: 8 warps, 64-feature slices;
//  * at least 6144: 8 warps, 32-feature slices;
//  * narrower outputs: 16 warps per CTA (few CTAs: more warps per SM), with
//    32-feature slices, or 16 when that would leave fewer than 100 CTAs.
// ring = shared-memory stages: as many as the budget allows once the CTAs are
// spread over the SMs.
int gemv_plan(int64_t M, int64_t K, int64_t N, int64_t G, int F_req, int W_req, int ring_req, GemvPlan* gp) {
  AWQB_REQUIRE(M >= 1 && M <= kGemvMaxM, kInvalidArgument, "small-batch path takes 1..%d rows (M=%lld)",
               kGemvMaxM, (long long)M);
  AWQB_REQUIRE(F_req == 0 || F_req == 16 || F_req == 32 || F_req == 64, kInvalidArgument,
               "feature slice %d not built (16, 32 or 64)", F_req);
  AWQB_REQUIRE(W_req == 0 || W_req == 8 || W_req == 16, kInvalidArgument, "compute warps %d not built (8 or 16)",
               W_req);
  AWQB_REQUIRE(ring_req >= 0 && ring_req <= 16, kInvalidArgument, "ring depth %d out of range (1..16, 0 = default)",
               ring_req);
  const int sm = device_sm_count();
  gp->MT = M <= 8 ? 8 : M <= 16 ? 16 : 32;
  gp->gpb = groups_per_block((int)G);
  int W = W_req, F = F_req;
  if (W == 0 && F == 0) {
    if (M > 8) {
      if (M <= 16 && N < 2048)
        W = 16, F = 16;  // few slices: more warps per CTA
      else
        W = 8, F = (N >= 6144 && M <= 16) ? 64 : 32;
    } else if (N >= 16384) {
      W = 8, F = 64;
    } else if (N >= 6144) {
      W = 8, F = 32;
    } else {
      W = 16, F = (N + 31) / 32 < 100 ? 16 : 32;
    }
  }
  if (W == 0) W = (F == 16) ? 16 : (F == 64 || N >= 6144 || M > 8) ? 8 : 16;
  if (F == 0) F = (W == 16) ? ((N + 31) / 32 < 100 ? 16 : 32) : 32;
  AWQB_REQUIRE(gemv_built(F, W), kUnsupported, "small-batch kernel with %d-feature slices and %d warps not built",
               F, W);
  const int64_t sb = gemv_stage_bytes_rt(F, W, gp->gpb, (int)M);
  AWQB_REQUIRE(sb > 0, kUnsupported, "no small-batch kernel for this configuration");
  AWQB_REQUIRE(kGemvSmemFixed + 2 * sb <= 227 * 1024 || (F_req > 0 && ring_req == 1), kUnsupported,
               "small-batch stages of %lld bytes do not fit twice in shared memory", (long long)sb);
  gp->F = F;
  gp->W = W;
  gp->ctas = (N + F - 1) / F;
  gp->kb_real = (int)((K + kBlockK - 1) / kBlockK);
  gp->stages = (gp->kb_real + W - 1) / W;
  if (ring_req > 0) {
    gp->ring = ring_req;
  } else {
    const int64_t per_sm = (gp->ctas + sm - 1) / sm;
    const int64_t budget = per_sm == 1 ? kGemvSmemAlone : kGemvSmemPerSm / per_sm;
    int64_t r = (budget - kGemvSmemFixed) / sb;
    // up to 8 rows, three stages are as fast or faster than deeper rings on
    // every Llama-3-8B decode shape (measured on B200: down at M = 1, 9.36 us
    // against 9.75 with four)
    r = std::max<int64_t>(2, std::min<int64_t>(gp->MT == 8 ? 3 : 16, r));
    gp->ring = (int)r;
  }
  if (gp->ring > gp->stages) gp->ring = std::max(1, gp->stages);
  // the epilogue's cross-warp reduction reuses the ring
  const int64_t red = (int64_t)W * F * gp->MT * 4;
  while ((int64_t)gp->ring * sb < red) ++gp->ring;
  gp->smem = kGemvSmemFixed + (int64_t)gp->ring * sb;
  AWQB_REQUIRE(gp->smem <= 227 * 1024, kUnsupported, "small-batch ring of %d stages does not fit (%lld bytes)",
               gp->ring, (long long)gp->smem);
  return kOk;
}

int encode_4d(CUtensorMap* tm, CUtensorMapDataType dt, const void* base, const cuuint64_t (&gdim)[4],
              const cuuint64_t (&gstride)[3], const cuuint32_t (&box)[4]) {
  auto enc = tensor_map_encoder();
  AWQB_REQUIRE(enc != nullptr, kCudaError, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint32_t estride[4] = {1u, 1u, 1u, 1u};
  CUresult r = enc(tm, dt, 4, const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AWQB_REQUIRE(r == CUDA_SUCCESS, kCudaError, "cuTensorMapEncodeTiled (weights) failed (%d)", (int)r);
  return kOk;
}

// The four tensor maps of one small-batch launch (awqb_gemv.cuh).
int make_gemv_maps(const void* x, const void* blob, int64_t M, int64_t K, int64_t N, const GemvPlan& gp,
                   CUtensorMap* tw, CUtensorMap* ts, CUtensorMap* tz, CUtensorMap* tx) {
  const int64_t KB = blob_kblocks(K);
  const int64_t NT = (N + kBlockN - 1) / kBlockN;
  const int64_t BB = block_bytes_for_gpb(gp.gpb);
  const uint8_t* b = static_cast<const uint8_t*>(blob);
  const int zw = gp.F / 8 < 4 ? 4 : gp.F / 8;
  {
    const cuuint64_t gdim[4] = {512, 4, (cuuint64_t)KB, (cuuint64_t)NT};
    const cuuint64_t gstr[3] = {2048, (cuuint64_t)BB, (cuuint64_t)(KB * BB)};
    const cuuint32_t box[4] = {(cuuint32_t)(4 * gp.F), 4, (cuuint32_t)gp.W, 1};
    int st = encode_4d(tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, b, gdim, gstr, box);
    if (st != kOk) return st;
  }
  {
    const cuuint64_t gdim[4] = {128, (cuuint64_t)gp.gpb, (cuuint64_t)KB, (cuuint64_t)NT};
    const cuuint64_t gstr[3] = {256, (cuuint64_t)BB, (cuuint64_t)(KB * BB)};
    const cuuint32_t box[4] = {(cuuint32_t)gp.F, (cuuint32_t)gp.gpb, (cuuint32_t)gp.W, 1};
    int st = encode_4d(ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, b + scale_off(), gdim, gstr, box);
    if (st != kOk) return st;
  }
  {
    const cuuint64_t gdim[4] = {16, (cuuint64_t)gp.gpb, (cuuint64_t)KB, (cuuint64_t)NT};
    const cuuint64_t gstr[3] = {64, (cuuint64_t)BB, (cuuint64_t)(KB * BB)};
    const cuuint32_t box[4] = {(cuuint32_t)zw, (cuuint32_t)gp.gpb, (cuuint32_t)gp.W, 1};
    int st = encode_4d(tz, CU_TENSOR_MAP_DATA_TYPE_UINT32, b + zero_off(gp.gpb), gdim, gstr, box);
    if (st != kOk) return st;
  }
  {
    auto enc = tensor_map_encoder();
    AWQB_REQUIRE(enc != nullptr, kCudaError, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t gdim[3] = {32, (cuuint64_t)M, (cuuint64_t)(K / 32)};
    const cuuint64_t gstr[2] = {(cuuint64_t)K * 2, 64};
    const cuuint32_t box[3] = {32, (cuuint32_t)M, (cuuint32_t)(4 * gp.W)};
    const cuuint32_t estride[3] = {1u, 1u, 1u};
    CUresult r = enc(tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(x), gdim, gstr, box, estride,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AWQB_REQUIRE(r == CUDA_SUCCESS, kCudaError, "cuTensorMapEncodeTiled (activations) failed (%d)", (int)r);
  }
  return kOk;
}

template <typename T, int F, int MT, int GPB, int W>
int gemv_launch_t(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tz, const CUtensorMap& tx,
                  const GemvParams& p, const GemvPlan& gp, cudaStream_t stream) {
  using Cfg = GemvCfg<F, MT, GPB, W>;
  auto kern = awq_gemv_kernel<T, F, MT, GPB, W>;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  AWQB_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    AWQB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gp.ctas);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = (size_t)gp.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AWQB_CUDA(cudaLaunchKernelEx(&cfg, kern, tw, ts, tz, tx, p));
  return kOk;
}

template <typename T, int F, int MT, int W>
int gemv_launch_g(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tz, const CUtensorMap& tx,
                  const GemvParams& p, const GemvPlan& gp, cudaStream_t s) {
  switch (gp.gpb) {
    case 1: return gemv_launch_t<T, F, MT, 1, W>(tw, ts, tz, tx, p, gp, s);
    case 2: return gemv_launch_t<T, F, MT, 2, W>(tw, ts, tz, tx, p, gp, s);
    case 4: return gemv_launch_t<T, F, MT, 4, W>(tw, ts, tz, tx, p, gp, s);
  }
  AWQB_REQUIRE(false, kUnsupported, "groups per block %d not built", gp.gpb);
  return kUnsupported;
}

template <typename T, int MT>
int gemv_launch_m(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tz, const CUtensorMap& tx,
                  const GemvParams& p, const GemvPlan& gp, cudaStream_t s) {
  if (gp.W == 16 && gp.F == 16) return gemv_launch_g<T, 16, MT, 16>(tw, ts, tz, tx, p, gp, s);
  if (gp.W == 16 && gp.F == 32) return gemv_launch_g<T, 32, MT, 16>(tw, ts, tz, tx, p, gp, s);
  if (gp.W == 8 && gp.F == 32) return gemv_launch_g<T, 32, MT, 8>(tw, ts, tz, tx, p, gp, s);
  if (gp.W == 8 && gp.F == 64) return gemv_launch_g<T, 64, MT, 8>(tw, ts, tz, tx, p, gp, s);
  AWQB_REQUIRE(false, kUnsupported, "small-batch kernel F=%d W=%d not built", gp.F, gp.W);
  return kUnsupported;
}

template <typename T>
int gemv_launch(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tz, const CUtensorMap& tx,
                const GemvParams& p, const GemvPlan& gp, cudaStream_t s) {
  if (gp.MT == 8) return gemv_launch_m<T, 8>(tw, ts, tz, tx, p, gp, s);
  if (gp.MT == 16) return gemv_launch_m<T, 16>(tw, ts, tz, tx, p, gp, s);
  return gemv_launch_m<T, 32>(tw, ts, tz, tx, p, gp, s);
}

// y = x * dequant(blob) (+ bias) for 1 <= M <= kGemvMaxM; sizes already
// validated by make_plan, pointers by the caller.
struct TpExchange;
void gemv_set_tp(GemvParams* p, const TpExchange* tp, int64_t M, int64_t N);

int gemv_impl(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype, const void* blob,
              const void* bias, void* y, int F_req, int W_req, int ring_req, bool silu, void* stream,
              const TpExchange* tp = nullptr) {
  GemvPlan gp;
  int st = gemv_plan(M, K, N, G, F_req, W_req, ring_req, &gp);
  if (st != kOk) return st;
  AWQB_REQUIRE(K % 32 == 0, kUnsupported, "K=%lld must be a multiple of 32", (long long)K);
  uint32_t* err = device_err_ptr();
  AWQB_REQUIRE(err != nullptr, kCudaError, "cannot resolve the device error word");
  CUtensorMap tw, ts, tz, tx;
  st = make_gemv_maps(x, blob, M, K, N, gp, &tw, &ts, &tz, &tx);
  if (st != kOk) return st;
  GemvParams p{};
  p.bias = bias;
  p.y = y;
  p.ldy = silu ? N / 2 : N;
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.K = (int32_t)K;
  p.kb_real = gp.kb_real;
  p.stages = gp.stages;
  p.ring = gp.ring;
  p.silu_mul = silu ? 1 : 0;
  p.err = err;
  if (tp != nullptr) gemv_set_tp(&p, tp, M, N);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == AWQB_DTYPE_F16) return gemv_launch<__half>(tw, ts, tz, tx, p, gp, s);
  return gemv_launch<__nv_bfloat16>(tw, ts, tz, tx, p, gp, s);
}

// Reduce-scatter + all-gather once the all-to-all traffic (world x the
// result, in 8-byte words) outweighs the extra hop: from 4 ranks and 8 rows.
bool tp_use_rsag(const TpExchange* tp, int64_t M) {
  return tp->mode == 2 || (tp->mode == 0 && tp->world >= 4 && M >= 8);
}

void gemv_set_tp(GemvParams* p, const TpExchange* tp, int64_t M, int64_t N) {
  p->tp_world = tp->world;
  p->tp_rank = tp->rank;
  p->tp_rows = (int32_t)tp->rows;
  p->tp_half = tp->half_words;
  p->tp_fhalf = tp->final_half;
  for (int r = 0; r < tp->world; ++r) {
    p->tp_land[r] = tp->land(r);
    p->tp_final[r] = tp->final_words(r);
  }
  p->tp_epoch = tp->epoch();
  p->tp_rsag = tp_use_rsag(tp, M) ? 1 : 0;
  (void)N;
}

int gemm_impl(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
              const void* blob, const void* bias, void* y, void* workspace,
              int64_t workspace_bytes, int ntok, int64_t ctas, void* stream,
              const TpExchange* tp = nullptr, bool silu = false) {
  AWQB_REQUIRE(dtype == AWQB_DTYPE_F16 || dtype == AWQB_DTYPE_BF16, kInvalidArgument,
               "dtype %d is not fp16 (0) or bf16 (1)", dtype);
  AWQB_REQUIRE(!silu || N % 16 == 0, kInvalidArgument,
               "fused SiLU-and-mul needs N = 2 * intermediate with intermediate a multiple of 8 (N=%lld)",
               (long long)N);
  Plan pl;
  int st = make_plan(M, K, N, G, ntok, ctas, &pl, !silu, tp != nullptr);
  if (st != kOk) return st;
  if (M == 0) return kOk;
  AWQB_REQUIRE(x != nullptr && blob != nullptr && y != nullptr, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(((uintptr_t)x & 15) == 0, kInvalidArgument, "x must be 16-byte aligned");
  AWQB_REQUIRE(((uintptr_t)blob & 15) == 0, kInvalidArgument, "blob must be 16-byte aligned");
  // Decode batches take the small-batch kernel (no workspace) unless a token
  // tile or CTA count was forced, or the call is the fused all-reduce.
  if (ntok == 0 && ctas <= 0 && gemv_takes(M, K, N)) {
    if (tp != nullptr) {
      AWQB_REQUIRE(tp->opened, kInvalidArgument, "exchange not opened (awqb_tp_exchange_open)");
      AWQB_REQUIRE(M <= tp->rows && N <= tp->max_n, kInvalidArgument,
                   "fused all-reduce sized for M <= %lld, N <= %lld (got M=%lld, N=%lld)", (long long)tp->rows,
                   (long long)tp->max_n, (long long)M, (long long)N);
    }
    return gemv_impl(x, M, K, N, G, dtype, blob, bias, y, 0, 0, 0, silu, stream, tp);
  }
  AWQB_REQUIRE(workspace != nullptr && ((uintptr_t)workspace & 255) == 0, kInvalidArgument,
               "workspace must be non-null and 256-byte aligned");
  AWQB_REQUIRE(workspace_bytes >= pl.cnt_bytes + pl.part_bytes, kInvalidArgument,
               "workspace too small: %lld < %lld bytes", (long long)workspace_bytes,
               (long long)(pl.cnt_bytes + pl.part_bytes));
  uint32_t* err = device_err_ptr();
  AWQB_REQUIRE(err != nullptr, kCudaError, "cannot resolve the device error word");

  CUtensorMap tm;
  int is3d = 0;
  st = make_x_tensor_map(&tm, x, M, K, pl.ntok, 2 * stage_blocks(pl.ntok), &is3d);
  if (st != kOk) return st;

  GemmParams p{};
  p.blob = static_cast<const uint8_t*>(blob);
  p.bias = bias;
  p.y = y;
  p.ldy = silu ? N / 2 : N;
  p.silu_mul = silu ? 1 : 0;
  p.num_valid = 0;
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.K = (int32_t)K;
  p.NT = pl.NT;
  p.KB = pl.KB;
  p.MT = pl.MT;
  p.ws_cnt = static_cast<int32_t*>(workspace);
  p.ws_part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + pl.cnt_bytes);
  p.err = err;
  p.x3d = is3d;
  p.group_m = raster_group_m(K, N, p.tile_expert != nullptr);
  p.cluster_s = pl.cluster_s;
  if (tp != nullptr) {
    AWQB_REQUIRE(tp->opened, kInvalidArgument, "exchange not opened (awqb_tp_exchange_open)");
    AWQB_REQUIRE(M <= tp->rows && N <= tp->max_n, kInvalidArgument,
                 "fused all-reduce sized for M <= %lld, N <= %lld (got M=%lld, N=%lld)", (long long)tp->rows,
                 (long long)tp->max_n, (long long)M, (long long)N);
    p.tp_world = tp->world;
    p.tp_rank = tp->rank;
    p.tp_rows = (int32_t)tp->rows;
    p.tp_half = tp->half_words;
    p.tp_fhalf = tp->final_half;
    for (int r = 0; r < tp->world; ++r) {
      p.tp_land[r] = tp->land(r);
      p.tp_final[r] = tp->final_words(r);
    }
    p.tp_epoch = tp->epoch();
    // reduce-scatter + all-gather is implemented in the cluster split-K finale
    p.tp_rsag = (pl.cluster_s > 1 && tp_use_rsag(tp, M)) ? 1 : 0;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == AWQB_DTYPE_F16) return launch_n<__half>(tm, p, pl, true, s);
  return launch_n<__nv_bfloat16>(tm, p, pl, true, s);
}

}  // namespace
}  // namespace awqb

using namespace awqb;

// Workspace sizes are those of the stream-K plan, which covers every launch the
// same arguments can make (cluster split-K needs no partials; fused SiLU-and-mul
// and the fused all-reduce use the same or a cluster plan).
extern "C" int awqb_gemm_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t G,
                                         int64_t* bytes) {
  Plan pl;
  int st = make_plan(M, K, N, G, 0, 0, &pl, false);
  if (st != kOk) return st;
  AWQB_REQUIRE(bytes != nullptr, kInvalidArgument, "bytes is null");
  *bytes = pl.cnt_bytes + pl.part_bytes;
  return kOk;
}

extern "C" int awqb_gemm_workspace_bytes_ex(int64_t M, int64_t K, int64_t N, int64_t G, int ntok,
                                            int64_t ctas, int64_t* bytes) {
  Plan pl;
  int st = make_plan(M, K, N, G, ntok, ctas, &pl, false);
  if (st != kOk) return st;
  AWQB_REQUIRE(bytes != nullptr, kInvalidArgument, "bytes is null");
  *bytes = pl.cnt_bytes + pl.part_bytes;
  return kOk;
}

extern "C" int awqb_gemm_plan(int64_t M, int64_t K, int64_t N, int64_t G, int ntok, int64_t ctas,
                              int* ntok_out, int64_t* ctas_out, int* cluster_out) {
  Plan pl;
  int st = make_plan(M, K, N, G, ntok, ctas, &pl, true);
  if (st != kOk) return st;
  AWQB_REQUIRE(ntok_out != nullptr && ctas_out != nullptr && cluster_out != nullptr, kInvalidArgument,
               "null output pointer");
  if (ntok == 0 && ctas <= 0 && gemv_takes(M, K, N)) {
    GemvPlan gp;
    st = gemv_plan(M, K, N, G, 0, 0, 0, &gp);
    if (st != kOk) return st;
    *ntok_out = gp.MT;
    *ctas_out = gp.ctas;
    *cluster_out = 0;
    return kOk;
  }
  *ntok_out = pl.ntok;
  *ctas_out = pl.ctas;
  *cluster_out = pl.cluster_s;
  return kOk;
}

extern "C" int awqb_gemm_silu_mul(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                                  const void* blob, const void* bias, void* y, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  return awqb::gemm_impl(x, M, K, N, G, dtype, blob, bias, y, workspace, workspace_bytes, 0, 0, stream, nullptr,
                         true);
}

extern "C" int awqb_gemm(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                         const void* blob, const void* bias, void* y, void* workspace,
                         int64_t workspace_bytes, void* stream) {
  return gemm_impl(x, M, K, N, G, dtype, blob, bias, y, workspace, workspace_bytes, 0, 0, stream);
}

extern "C" int awqb_gemm_ex(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                            const void* blob, const void* bias, void* y, void* workspace,
                            int64_t workspace_bytes, int ntok, int64_t ctas, void* stream) {
  return gemm_impl(x, M, K, N, G, dtype, blob, bias, y, workspace, workspace_bytes, ntok, ctas,
                   stream);
}

extern "C" int awqb_gemv_ex(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                            const void* blob, const void* bias, void* y, int features_per_cta, int warps, int ring,
                            int silu_mul, void* stream) {
  Plan pl;
  int st = make_plan(M, K, N, G, 0, 0, &pl, false);
  if (st != kOk) return st;
  AWQB_REQUIRE(dtype == AWQB_DTYPE_F16 || dtype == AWQB_DTYPE_BF16, kInvalidArgument,
               "dtype %d is not fp16 (0) or bf16 (1)", dtype);
  AWQB_REQUIRE(!silu_mul || N % 16 == 0, kInvalidArgument, "fused SiLU-and-mul needs N %% 16 == 0");
  AWQB_REQUIRE(x != nullptr && blob != nullptr && y != nullptr, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)blob & 15) == 0, kInvalidArgument,
               "x and blob must be 16-byte aligned");
  return gemv_impl(x, M, K, N, G, dtype, blob, bias, y, features_per_cta, warps, ring, silu_mul != 0, stream);
}

// ---------------------------------------------------------------------------
// GEMM without any caller-provided or library-allocated workspace.
//
// Some callers have no way to hand this library device memory: a host that
// manages every device byte through its own arena and does not let plug-ins
// allocate, or code that must not call cudaMalloc at all because it may run
// while a CUDA graph is being captured or on a latency-critical path where the
// implicit synchronisation of an allocation is not acceptable. For them the
// split-K scratch (tile counters + fp32 partial tiles) lives in a fixed array
// compiled into this library. Every GPU that loads the library keeps those
// kNoAllocScratchBytes for the life of the process.
namespace awqb {
namespace {

constexpr int64_t kNoAllocScratchBytes = 16ll << 20;  // 16 MiB: every M <= 64 fits
__device__ __align__(256) uint8_t g_awqb_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array for the current device. The array's name
// is only a host-side stand-in, so the address is looked up once per device,
// with that device current, and cached.
int noalloc_scratch(uint8_t** out) {
  static uint8_t* ptrs[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  AWQB_CUDA(cudaGetDevice(&dev));
  AWQB_REQUIRE(dev >= 0 && dev < kMaxDevices, kUnsupported, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    AWQB_CUDA(cudaGetSymbolAddress(&p, g_awqb_noalloc_scratch));
    ptrs[dev] = static_cast<uint8_t*>(p);
  }
  *out = ptrs[dev];
  return kOk;
}

}  // namespace
}  // namespace awqb

extern "C" int64_t awqb_gemm_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int awqb_gemm_noalloc(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                                 const void* blob, const void* bias, void* y, void* stream) {
  Plan pl;
  int st = make_plan(M, K, N, G, 0, 0, &pl, true);
  if (st != kOk) return st;
  if (M == 0) return kOk;
  const int64_t need = pl.cnt_bytes + pl.part_bytes;
  AWQB_REQUIRE(need <= kNoAllocScratchBytes, kUnsupported,
               "M=%lld K=%lld N=%lld needs %lld bytes of split-K scratch; the no-allocation entry "
               "point has %lld (every M <= 64 fits). Use awqb_gemm with a workspace instead.",
               (long long)M, (long long)K, (long long)N, (long long)need, (long long)kNoAllocScratchBytes);
  uint8_t* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st != kOk) return st;
  // The array keeps whatever the previous call left; the tile counters must
  // start at zero (the partial tiles are always written before they are read).
  AWQB_CUDA(cudaMemsetAsync(scratch, 0, (size_t)pl.cnt_bytes, static_cast<cudaStream_t>(stream)));
  return gemm_impl(x, M, K, N, G, dtype, blob, bias, y, scratch, kNoAllocScratchBytes, 0, 0, stream);
}

extern "C" int awqb_device_error(uint32_t* out) {
  AWQB_REQUIRE(out != nullptr, kInvalidArgument, "out is null");
  AWQB_CUDA(cudaDeviceSynchronize());
  AWQB_CUDA(cudaMemcpyFromSymbol(out, g_awqb_err, sizeof(uint32_t)));
  return kOk;
}

extern "C" int awqb_clear_device_error(void) {
  const uint32_t zero = 0;
  AWQB_CUDA(cudaDeviceSynchronize());
  AWQB_CUDA(cudaMemcpyToSymbol(g_awqb_err, &zero, sizeof(uint32_t)));
  return kOk;
}

// ---------------------------------------------------------------------------
// Grouped GEMM over expert-sorted rows (MoE). Row block b (ntok rows) uses the
// weights of expert block_expert[b]; only the first *num_post_pad rows are
// computed (a device value, so the call needs no host sync and can be
// captured). With row_map, output row = row_map[r] and rows mapping to
// >= num_valid (padding) are skipped; with row_scale the output row is scaled
// by row_scale[output row] (the router weight, fused.py:183-196 with
// MUL_ROUTED_WEIGHT, triton/fused_moe.py:276-278).
namespace awqb {
namespace {
int64_t grouped_ctas(int64_t ctas) { return ctas > 0 ? ctas : device_sm_count(); }
}  // namespace
}  // namespace awqb

extern "C" int awqb_moe_grouped_workspace_bytes(int64_t rows_max, int64_t K, int64_t N, int64_t G,
                                                int ntok, int64_t* bytes) {
  Plan pl;
  int st = make_plan(rows_max, K, N, G, ntok, 0, &pl);
  if (st != kOk) return st;
  AWQB_REQUIRE(bytes != nullptr, kInvalidArgument, "bytes is null");
  const int64_t c = grouped_ctas(0);
  *bytes = pl.cnt_bytes + c * 2 * 128 * (int64_t)pl.ntok * 4;
  return kOk;
}

namespace awqb {
namespace {
int grouped_impl(const void* x_sorted, int64_t rows_max, int64_t K, int64_t N,
                                     int64_t G, int dtype, const void* blobs, int64_t blob_stride,
                                     const int32_t* block_expert, const int32_t* num_post_pad,
                                     int ntok, const int32_t* row_map, const float* row_scale,
                                     int64_t num_valid, void* y, int64_t ldy, void* workspace,
                                     int64_t workspace_bytes, void* stream, bool silu) {
  AWQB_REQUIRE(dtype == AWQB_DTYPE_F16 || dtype == AWQB_DTYPE_BF16, kInvalidArgument,
               "dtype %d is not fp16 (0) or bf16 (1)", dtype);
  AWQB_REQUIRE(ntok == 16 || ntok == 32 || ntok == 64 || ntok == 128 || ntok == 256,
               kInvalidArgument, "block size %d must equal a built token tile", ntok);
  Plan pl;
  int st = make_plan(rows_max, K, N, G, ntok, 0, &pl);
  if (st != kOk) return st;
  if (rows_max == 0) return kOk;
  pl.ctas = grouped_ctas(0);
  pl.part_bytes = pl.ctas * 2 * 128 * (int64_t)pl.ntok * 4;
  AWQB_REQUIRE(2 * pl.ctas * pl.ctas * (pl.KB / stage_blocks(pl.ntok)) < (1ll << 31), kUnsupported,
               "K=%lld too large for %lld CTAs", (long long)K, (long long)pl.ctas);
  AWQB_REQUIRE(x_sorted && blobs && block_expert && num_post_pad && y, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(((uintptr_t)x_sorted & 15) == 0 && ((uintptr_t)blobs & 15) == 0 && blob_stride % 16 == 0,
               kInvalidArgument, "x_sorted, blobs and blob_stride must be 16-byte aligned");
  AWQB_REQUIRE(ldy >= (silu ? N / 2 : N), kInvalidArgument, "ldy too small");
  AWQB_REQUIRE(workspace != nullptr && ((uintptr_t)workspace & 255) == 0, kInvalidArgument,
               "workspace must be non-null and 256-byte aligned");
  AWQB_REQUIRE(workspace_bytes >= pl.cnt_bytes + pl.part_bytes, kInvalidArgument,
               "workspace too small: %lld < %lld bytes", (long long)workspace_bytes,
               (long long)(pl.cnt_bytes + pl.part_bytes));
  uint32_t* err = device_err_ptr();
  AWQB_REQUIRE(err != nullptr, kCudaError, "cannot resolve the device error word");
  CUtensorMap tm;
  int is3d = 0;
  st = make_x_tensor_map(&tm, x_sorted, rows_max, K, pl.ntok, 2 * stage_blocks(pl.ntok), &is3d);
  if (st != kOk) return st;
  GemmParams p{};
  p.blob = static_cast<const uint8_t*>(blobs);
  p.blob_stride = blob_stride;
  p.tile_expert = block_expert;
  p.rows_valid = num_post_pad;
  p.y = y;
  p.ldy = ldy;
  p.silu_mul = silu ? 1 : 0;
  p.row_map = row_map;
  p.row_scale = row_scale;
  p.num_valid = (int32_t)num_valid;
  p.M = (int32_t)rows_max;
  p.N = (int32_t)N;
  p.K = (int32_t)K;
  p.NT = pl.NT;
  p.KB = pl.KB;
  p.MT = pl.MT;
  p.ws_cnt = static_cast<int32_t*>(workspace);
  p.ws_part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + pl.cnt_bytes);
  p.err = err;
  p.x3d = is3d;
  p.group_m = raster_group_m(K, N, p.tile_expert != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == AWQB_DTYPE_F16) return launch_n<__half>(tm, p, pl, false, s);
  return launch_n<__nv_bfloat16>(tm, p, pl, false, s);
}
}  // namespace
}  // namespace awqb

extern "C" int awqb_moe_grouped_gemm(const void* x_sorted, int64_t rows_max, int64_t K, int64_t N,
                                     int64_t G, int dtype, const void* blobs, int64_t blob_stride,
                                     const int32_t* block_expert, const int32_t* num_post_pad,
                                     int ntok, const int32_t* row_map, const float* row_scale,
                                     int64_t num_valid, void* y, int64_t ldy, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  return awqb::grouped_impl(x_sorted, rows_max, K, N, G, dtype, blobs, blob_stride, block_expert, num_post_pad,
                            ntok, row_map, row_scale, num_valid, y, ldy, workspace, workspace_bytes, stream, false);
}

extern "C" int awqb_moe_grouped_gemm_silu_mul(const void* x_sorted, int64_t rows_max, int64_t K, int64_t N,
                                              int64_t G, int dtype, const void* blobs, int64_t blob_stride,
                                              const int32_t* block_expert, const int32_t* num_post_pad,
                                              int ntok, void* y, int64_t ldy, void* workspace,
                                              int64_t workspace_bytes, void* stream) {
  using namespace awqb;
  AWQB_REQUIRE(N % 16 == 0, kInvalidArgument, "fused SiLU-and-mul needs N a multiple of 16 (N=%lld)",
               (long long)N);
  AWQB_REQUIRE(ldy >= N / 2, kInvalidArgument, "ldy < N / 2");
  return grouped_impl(x_sorted, rows_max, K, N, G, dtype, blobs, blob_stride, block_expert, num_post_pad, ntok,
                      nullptr, nullptr, 0, y, ldy, workspace, workspace_bytes, stream, true);
}

// ---------------------------------------------------------------------------
// Fused row-parallel GEMM + all-reduce over peer memory.
extern "C" int awqb_tp_exchange_create(int rank, int world, int64_t max_rows, int64_t max_n, void** ctx) {
  using namespace awqb;
  AWQB_REQUIRE(ctx != nullptr, kInvalidArgument, "ctx is null");
  AWQB_REQUIRE(world >= 1 && world <= 8 && rank >= 0 && rank < world, kInvalidArgument,
               "rank %d / world %d (1..8 ranks)", rank, world);
  AWQB_REQUIRE(max_rows >= 1 && max_rows <= 256 && max_n >= 8 && max_n % 8 == 0, kInvalidArgument,
               "max_rows must be 1..256 and max_n a positive multiple of 8");
  auto* t = new TpExchange();
  t->rank = rank;
  t->world = world;
  t->rows = max_rows;
  t->max_n = max_n;
  t->half_words = (int64_t)world * max_rows * max_n;
  t->final_half = max_rows * max_n;
  cudaError_t e = cudaGetDevice(&t->device);
  if (e == cudaSuccess) e = cudaMalloc(&t->local, (size_t)t->total_bytes());
  if (e == cudaSuccess) e = cudaMemset(t->local, 0, (size_t)t->total_bytes());
  if (e != cudaSuccess) {
    if (t->local) cudaFree(t->local);
    delete t;
    AWQB_CUDA(e);
  }
  t->base[rank] = t->local;
  *ctx = t;
  return kOk;
}

extern "C" int awqb_tp_exchange_handle(void* ctx, void* handle_out) {
  using namespace awqb;
  AWQB_REQUIRE(ctx != nullptr && handle_out != nullptr, kInvalidArgument, "null pointer");
  auto* t = static_cast<TpExchange*>(ctx);
  cudaIpcMemHandle_t h;
  AWQB_CUDA(cudaIpcGetMemHandle(&h, t->local));
  memcpy(handle_out, &h, sizeof(h));
  return kOk;
}

extern "C" int awqb_tp_exchange_open(void* ctx, const void* handles) {
  using namespace awqb;
  AWQB_REQUIRE(ctx != nullptr && handles != nullptr, kInvalidArgument, "null pointer");
  auto* t = static_cast<TpExchange*>(ctx);
  AWQB_REQUIRE(!t->opened, kInvalidArgument, "exchange already opened");
  for (int r = 0; r < t->world; ++r) {
    if (r == t->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != t->rank && t->base[q]) cudaIpcCloseMemHandle(t->base[q]);
      AWQB_CUDA(e);
    }
    t->base[r] = ptr;
  }
  t->opened = true;
  return kOk;
}

extern "C" int awqb_tp_exchange_handle_bytes(int64_t* bytes) {
  using namespace awqb;
  AWQB_REQUIRE(bytes != nullptr, kInvalidArgument, "bytes is null");
  *bytes = (int64_t)sizeof(cudaIpcMemHandle_t);
  return kOk;
}

extern "C" int awqb_tp_exchange_set_mode(void* ctx, int mode) {
  using namespace awqb;
  AWQB_REQUIRE(ctx != nullptr, kInvalidArgument, "ctx is null");
  AWQB_REQUIRE(mode >= 0 && mode <= 2, kInvalidArgument, "mode must be 0 (auto), 1 or 2");
  static_cast<TpExchange*>(ctx)->mode = mode;
  return kOk;
}

extern "C" int awqb_tp_exchange_destroy(void* ctx) {
  using namespace awqb;
  if (ctx == nullptr) return kOk;
  auto* t = static_cast<TpExchange*>(ctx);
  cudaDeviceSynchronize();
  for (int r = 0; r < t->world; ++r)
    if (r != t->rank && t->base[r]) cudaIpcCloseMemHandle(t->base[r]);
  if (t->local) cudaFree(t->local);
  delete t;
  return kOk;
}

extern "C" int awqb_gemm_allreduce(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                                   const void* blob, const void* bias, void* y, void* workspace,
                                   int64_t workspace_bytes, void* ctx, void* stream) {
  using namespace awqb;
  AWQB_REQUIRE(ctx != nullptr, kInvalidArgument, "ctx is null");
  return gemm_impl(x, M, K, N, G, dtype, blob, bias, y, workspace, workspace_bytes, 0, 0, stream,
                   static_cast<const TpExchange*>(ctx));
}
