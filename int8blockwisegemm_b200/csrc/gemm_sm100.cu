// Persistent grouped INT8 GEMMs on the 5th-generation tensor cores (sm_100a).
//
// One kernel template serves
//   * the hybrid blockwise GEMM (reference
//     csrc/int8_hybrid_grouped_gemm.cu:218-479): for every 128-deep K-tile
//     (or quant block of several K-tiles) the int32 partial product is
//     multiplied by Q_A[s, qb] * Q_B[e, n/64, qb] and added to an int32
//     running sum; at the end out = dtype(float(W) * (F_A[s,0] * F_B[e,n/64,0]))
//     (+ bias, added after the rounded product, for the _bias variants);
//   * the per-tensor grouped GEMM (csrc/int8_grouped_gemm.cu:35-47,193-219):
//     out = dtype(float(sum_k a*b) * alpha) with alpha per tensor, or
//     per-token x per-expert (extension).
//
// Structure (one CTA per SM; tiles of 128 rows x 256 columns):
//   warp 0      TMA producer: A tile [128 rows x 128 K] and B tile
//               [BN x 128 K] per K-tile, 128-byte swizzle, into a STAGES-deep
//               shared-memory ring guarded by full/empty mbarriers.
//   warp 1      TMEM allocator + single-thread MMA issuer:
//               tcgen05.mma.cta_group::1.kind::i8, M=128, N=256, K=32, four
//               per K-tile, accumulating one quant block into one of two TMEM
//               accumulator buffers (256 columns each); tcgen05.commit frees
//               the smem stage and, at the end of a quant block, signals the
//               epilogue.
//   warps 2, 3  idle (they complete warpgroup 0, which hands its registers
//               to the epilogue through setmaxnreg)
//   warps 4..   epilogue: TMEM lane quadrant = warp % 4, column group =
//               (warp - 4) / 4.  Each thread owns one output row and 128
//               columns (8 epilogue warps, 232 registers a thread; CTA pairs:
//               16 warps of 64 columns at 112): tcgen05.ld the block partial
//               in 32-column chunks, release the TMEM buffer after the last
//               load, W += q * P (int32 IMAD); after the last block convert,
//               scale, round and store the row through shared-memory staging
//               and TMA tensor stores (rows beyond the expert are not
//               stored, so neighbouring experts are never overwritten).
//               The hybrid format costs one integer multiply-add per output
//               element per quant block, about the tensor-core rate at
//               128-deep blocks, so the epilogue's instruction issue, not the
//               MMA, sets the pace: fewer, wider warps issue fewer
//               per-block instructions for the same multiply-adds.
// Tiles: (expert, 128-row m-tile, BN-col n-tile), m-tile major, walked
// round-robin by the persistent CTAs; the per-expert m-tile prefix is built
// in shared memory from problem_sizes at kernel start (no host loop, no
// host synchronisation).
//
// K tiling follows the reference's CUTLASS 2.x iterators, which visit the
// partial residue tile first: K-tile kt covers [kt*128 - pad, (kt+1)*128 - pad)
// with pad = 128*ceil(K/128) - K; the TMA load of tile 0 starts at the
// negative column -pad and the out-of-range columns are zero-filled.
#include <algorithm>
#include <cstdlib>
#include <cudaTypedefs.h>
#include <type_traits>
#include <mutex>

#include "common.cuh"
#include "quant_math.cuh"

namespace i8moe {

static __device__ unsigned g_err_gemm;

int read_gemm_error(uint32_t* w, int clear) {
  unsigned v = 0;
  I8_CUDA(cudaMemcpyFromSymbol(&v, g_err_gemm, sizeof(v)));
  if (clear) {
    unsigned z = 0;
    I8_CUDA(cudaMemcpyToSymbol(g_err_gemm, &z, sizeof(z)));
  }
  *w = v;
  return I8MOE_OK;
}

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes == int8 elements per K-tile
constexpr int NACC = 2;
// Warps 0-3 (one warpgroup): TMA producer, MMA issuer, two idle; then the
// epilogue warps.  Launched at Epi::kRegsLaunch registers a thread, the
// first warpgroup gives registers back (setmaxnreg.dec to kRegsLow) and the
// epilogue warpgroups take them (setmaxnreg.inc to kRegsHigh); CTA pairs:
// 20 warps x 32 x 96 = 128 x 32 + 512 x 112 registers exactly.
constexpr int kEpiW0 = 4;
constexpr int kEpiWarps = 16;  // epilogue warps of the CTA-pair kernels

// The one-CTA store epilogue runs 8 wide epilogue warps instead: each
// thread owns one row and 128 accumulator columns (two 64-column
// weight-scale blocks).  Half as many warps issue half as many per-block
// instructions (barrier waits, fences, loop control) for the same int32
// multiply-adds, and at 232 registers a thread the 128 running sums fit
// beside a 32-column load.  12 warps x 32 x 168 = 128 x 40 + 256 x 232
// registers.  The fused SiLU epilogue keeps 16 warps of 64 columns: its
// per-tile SiLU / requant phase is latency-bound and wide warps made it
// slower (w13 at the default shape 336 against 314 us); so do CTA pairs.
template <int EPI, int CG>
struct Epi {
  static constexpr bool kWide = EPI == 0 && CG == 1;  // EPI 0: kEpiStore
  static constexpr int kWarps = kWide ? 8 : kEpiWarps;
  static constexpr int kCols = kWide ? 128 : 64;  // accumulator columns a thread
  static constexpr int kThreads = 32 * kEpiW0 + 32 * kWarps;
  static constexpr int kRegsLaunch = kWide ? 168 : 96;
  static constexpr int kRegsLow = kWide ? 40 : 32;
  static constexpr int kRegsHigh = kWide ? 232 : 112;
  static_assert(kThreads * kRegsLaunch == 32 * kEpiW0 * kRegsLow + 32 * kWarps * kRegsHigh,
                "register split must use exactly the registers the block is launched with");
  static_assert(kRegsLaunch * kThreads <= 65536, "register file");
};
constexpr int kMaxExperts = 1024;
constexpr int kTileABytes = BM * BK;
constexpr uint32_t kTmemCols = NACC * BN;
constexpr int kSmemLimit = 227 * 1024;  // dynamic shared memory per CTA on sm_100

// CG = 1: one CTA per 128 x 256 tile (tcgen05.mma.cta_group::1, M = 128),
//   every CTA streams A [128 x 128] and all of B [256 x 128] per K-tile.
// CG = 2: a cluster of two CTAs per 256 x 256 pair tile (cta_group::2,
//   M = 256): each CTA streams its own A rows and half of the B rows
//   (32 KB per K-tile instead of 48 KB), so the ring is five stages deep.
template <int CG>
struct Cfg {
  static constexpr int kStages = CG == 2 ? 5 : 3;
  static constexpr int kBRows = BN / CG;  // B rows this CTA loads per K-tile
  static constexpr int kTileBBytes = kBRows * BK;
  static constexpr uint32_t kIdesc = idesc_i8(BM * CG, BN);
};

enum GemmMode { kHybrid = 0, kPerTensor = 1 };
// Epilogue: store the scaled product, or (w13 only) SiLU(gate)*up + INT8
// requant of the intermediate activation.
enum GemmEpilogue { kEpiStore = 0, kEpiSiluQuant = 1 };

struct GemmParams {
  const int32_t* eo;   // [E+1]
  const int32_t* ps;   // [E, 3]
  const int32_t* so;   // [E] or null
  const int32_t* qa;
  const float* fa;
  const int32_t* qb;
  const float* fb;
  const float* bias;
  int bias_stride;
  const float* a_row_scale;
  const float* b_expert_scale;
  float alpha;
  void* out;
  int E, sum_m, N, K;
  int kt_total, k_pad, ktpq, nq;
  int q_stride, f_stride, nsb;
  int tile_m;
  int n_tiles;
  // kEpiSiluQuant: N is the w13 output width 2*n_act; the tile's B rows are
  // gate rows [n0, n0+128) and up rows [n_act+n0, +128)
  int n_act;
  int8_t* act_q;       // [sum_m, n_act] int8
  float* act_scale;    // [scale rows, kb_act] raw block scales (in the Q buffer)
  int kb_act;
};

template <int CG, int EPI>
struct SmemLayout {
  static constexpr int kStages = Cfg<CG>::kStages;
  static constexpr int kWarps = Epi<EPI, CG>::kWarps;
  static constexpr int kA = 0;
  static constexpr int kB = kA + kStages * kTileABytes;
  // per-epilogue-warp output staging (32 rows x 64 B, 64-byte swizzle; two
  // such buffers for the wide warps)
  static constexpr int kStg = kB + kStages * Cfg<CG>::kTileBBytes;  // 1024-B aligned
  static constexpr int kStgBufBytes = 32 * 64;
  static constexpr int kStgWarpBytes = Epi<EPI, CG>::kWide ? 2 * kStgBufBytes : kStgBufBytes;
  static constexpr int kBar = kStg + kWarps * kStgWarpBytes;  // 8-B aligned
  // full/empty ring, accumulator full/empty, final drain, and the two
  // row-group absmax barriers of the fused SiLU-quant epilogue
  static constexpr int kNumBars = 2 * kStages + 2 * NACC + 1 + 2;
  static constexpr int kMisc = kBar + kNumBars * 8;   // tmem base, abort flag
  static constexpr int kRed = kMisc + 16;             // absmax slots [2 groups][3]
  // per-epilogue-thread slots (Q_A, Q_B, Q_B(up) per tile parity; F_A, F_B,
  // F_B(up) of the current tile), then the per-expert tables: m-tile prefix,
  // scale-row offset, row count, first row
  static constexpr int kSlots = kRed + 32;
  static constexpr int kSlotArray = 4 * 32 * kWarps;
  static constexpr int kPrefix = kSlots + 9 * kSlotArray;
  static constexpr int bytes(int E) { return kPrefix + 4 * (E + 1) * 4 + 32; }
};

// The _bias epilogue as the reference evaluates it: the scaled accumulator
// rounded to fp32 first, then the bias added (a separate rounding, no FMA;
// int8_hybrid_grouped_gemm.cu:449-458 -- pinned by running the reference).
__device__ __forceinline__ float bias_epi(int32_t w, float f, float bias) {
  return __fadd_rn(__fmul_rn(static_cast<float>(w), f), bias);
}

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ void block_exclusive_scan(int* s, int n, int* s_tmp) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int per = (n + nt - 1) / nt;
  const int lo = tid * per;
  int local = 0;
  for (int i = 0; i < per; ++i)
    if (lo + i < n) local += s[lo + i];
  const int lane = tid & 31, warp = tid >> 5;
  int v = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) s_tmp[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (nt >> 5) ? s_tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_tmp[lane] = w;
  }
  __syncthreads();
  int prefix = v - local + (warp > 0 ? s_tmp[warp - 1] : 0);
  for (int i = 0; i < per; ++i) {
    if (lo + i < n) {
      const int x = s[lo + i];
      s[lo + i] = prefix;
      prefix += x;
    }
  }
  if (n > 0 && lo < n && lo + per >= n) s[n] = prefix;
  if (n == 0 && tid == 0) s[0] = 0;
  __syncthreads();
}

struct TileInfo {
  int e, mt, nt;
};

__device__ __forceinline__ TileInfo decode_tile(int t, const int* mt_prefix, int E, int n_tiles) {
  const int gm = t / n_tiles;
  TileInfo ti;
  ti.nt = t - gm * n_tiles;
  int lo = 0, hi = E;  // last e with mt_prefix[e] <= gm
  while (lo + 1 < hi) {
    const int mid = (lo + hi) >> 1;
    if (mt_prefix[mid] <= gm) lo = mid; else hi = mid;
  }
  ti.e = lo;
  ti.mt = gm - mt_prefix[lo];
  return ti;
}

// the tile's coordinates as seen by this CTA: with CTA pairs, mt_prefix
// counts pair tiles and the CTA of rank r owns m-tile 2 * (pair m-tile) + r
template <int CG>
__device__ __forceinline__ TileInfo decode_tile_cta(int t, const int* mt_prefix, int E,
                                                    int n_tiles, int rank) {
  TileInfo ti = decode_tile(t, mt_prefix, E, n_tiles);
  if (CG == 2) ti.mt = 2 * ti.mt + rank;
  return ti;
}

template <int MODE, bool HAS_BIAS, typename OutT, int EPI, int CG>
__global__ void __launch_bounds__((Epi<EPI, CG>::kThreads), 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO, const GemmParams p) {
  using SmemLayout = i8moe::SmemLayout<CG, EPI>;
  using EP = Epi<EPI, CG>;
  constexpr int kThreads = EP::kThreads;
  constexpr int kEW = EP::kWarps;     // epilogue warps
  constexpr bool kWide = EP::kWide;   // 128 accumulator columns a thread
  constexpr int STAGES = Cfg<CG>::kStages;
  constexpr int kTileBBytes = Cfg<CG>::kTileBBytes;
  constexpr uint32_t kIdesc = Cfg<CG>::kIdesc;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + SmemLayout::kBar;
  const uint32_t bar_empty = bar_full + STAGES * 8;
  const uint32_t bar_accf = bar_empty + STAGES * 8;
  const uint32_t bar_acce = bar_accf + NACC * 8;
  const uint32_t bar_final = bar_acce + NACC * 8;
  const uint32_t bar_red = bar_final + 8;  // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + SmemLayout::kMisc);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + SmemLayout::kMisc + 4);
  int* s_tmp = reinterpret_cast<int*>(smem + SmemLayout::kA);  // scratch before the first TMA
  int* mt_prefix = reinterpret_cast<int*>(smem + SmemLayout::kPrefix);
  int* so_prefix = mt_prefix + (p.E + 1);
  int* m_rows = so_prefix + (p.E + 1);
  int* e_row0 = m_rows + (p.E + 1);

  // ---- prologue: per-expert tables (tile prefix, scale rows, rows) ----
  // Kept in shared memory so a tile's coordinates resolve without global
  // loads on the epilogue's critical path.
  // Tiles are enumerated per CTA pair when CG == 2: mt_prefix then counts
  // pair tiles (two 128-row m-tiles each), and a CTA's own m-tile is
  // 2 * (pair m-tile) + its rank in the pair.
  const int rank = CG == 2 ? static_cast<int>(cluster_ctarank()) : 0;
  const int tile0 = CG == 2 ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int tstride = CG == 2 ? static_cast<int>(cluster_count_x()) : static_cast<int>(gridDim.x);
  for (int e = threadIdx.x; e < p.E; e += kThreads) {
    const int m = max(0, __ldg(p.ps + 3 * e));
    mt_prefix[e] = CG == 2 ? ((m + BM - 1) / BM + 1) / 2 : (m + BM - 1) / BM;
    so_prefix[e] = p.so ? __ldg(p.so + e) : (m + p.tile_m - 1) / p.tile_m;
    m_rows[e] = m;
    e_row0[e] = __ldg(p.eo + e);
  }
  if (threadIdx.x == 0) *s_abort = 0;
  if (threadIdx.x < 6) reinterpret_cast<unsigned*>(smem + SmemLayout::kRed)[threadIdx.x] = 0u;
  __syncthreads();
  block_exclusive_scan(mt_prefix, p.E, s_tmp);
  if (p.so == nullptr) block_exclusive_scan(so_prefix, p.E, s_tmp);
  const int total_tiles = mt_prefix[p.E] * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(bar_accf + 8 * a, 1);
      // released by every thread of the wide epilogue, else by lane 0 of
      // every epilogue warp (of both CTAs of a pair)
      mbar_init(bar_acce + 8 * a, kWide ? 32 * kEW : CG * kEW);
    }
    mbar_init(bar_final, 1);
    // absmax groups: all 16 epilogue warps (tile_m 128) or the 8 warps of
    // each 64-row half (tile_m 64)
    mbar_init(bar_red, p.tile_m == 64 ? kEW / 2 : kEW);
    mbar_init(bar_red + 8, p.tile_m == 64 ? kEW / 2 : kEW);
    mbar_fence_init();
  }
  // the other CTA of a pair signals this CTA's barriers: they must be
  // initialised before either CTA goes on
  if constexpr (CG == 2) cluster_sync();
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(smem_u32(s_tmem), kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(s_tmem), kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  // the pair's first CTA holds the ring's full barriers and the accumulator
  // empty barriers that both CTAs signal
  const uint32_t full0 = CG == 2 ? mapa_shared(bar_full, 0) : bar_full;
  const uint32_t acce0 = CG == 2 ? mapa_shared(bar_acce, 0) : bar_acce;

  if (warp < kEpiW0) {
  // register split, first warpgroup: gives registers back (the host checked
  // the launch count); each role's code sits inside its warpgroup's branch
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(EP::kRegsLow));
  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_phase[s] = 0;
      bool ok = true;
      for (int t = tile0; t < total_tiles && ok; t += tstride) {
        const TileInfo ti = decode_tile_cta<CG>(t, mt_prefix, p.E, p.n_tiles, rank);
        const int row0 = e_row0[ti.e] + ti.mt * BM;
        const int n0 = ti.nt * (EPI == kEpiSiluQuant ? 128 : BN);
        // CG == 2: an expert with an odd number of m-tiles leaves one CTA of
        // its last pair tile without rows; that CTA loads no A (its
        // accumulator rows are discarded) but still its half of B.
        const int mt_e = (m_rows[ti.e] + BM - 1) / BM;
        const bool own_ok = ti.mt < mt_e;
        const bool peer_ok = CG == 2 && (ti.mt ^ 1) < mt_e;
        const uint32_t tx = CG == 2 ? (own_ok + peer_ok) * kTileABytes + 2 * kTileBBytes
                                    : kTileABytes + kTileBBytes;
        // this CTA's B rows: store epilogue [n0 + 128*rank, +128) of the
        // tile; fused SiLU epilogue gate rows [n0, +128) (first CTA) and the
        // matching up rows [n_act + n0, +128) (second CTA)
        const int b_row = EPI == kEpiSiluQuant ? (rank ? p.n_act + n0 : n0) : n0 + 128 * rank;
        for (int kt = 0; kt < p.kt_total; ++kt) {
          if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1, s_abort, &g_err_gemm,
                         kErrProducerTimeout)) {
            ok = false;
            break;
          }
          const int kx = kt * BK - p.k_pad;
          const uint32_t b_dst = sbase + SmemLayout::kB + stage * kTileBBytes;
          const uint32_t a_dst = sbase + SmemLayout::kA + stage * kTileABytes;
          if constexpr (CG == 2) {
            if (rank == 0) mbar_arrive_expect_tx(bar_full + 8 * stage, tx);
            const uint32_t fb = full0 + 8 * stage;
            if (own_ok) tma_load_2d_pair(a_dst, &tmA, fb, kx, row0);
            tma_load_3d_pair(b_dst, &tmB, fb, kx, b_row, ti.e);
          } else {
            const uint32_t fb = bar_full + 8 * stage;
            mbar_arrive_expect_tx(fb, tx);
            tma_load_2d(a_dst, &tmA, fb, kx, row0);
            if (EPI == kEpiSiluQuant) {
              // gate rows [n0, n0+128) and the matching up rows [n_act+n0, +128)
              tma_load_3d(b_dst, &tmB, fb, kx, n0, ti.e);
              tma_load_3d(b_dst + kTileBBytes / 2, &tmB, fb, kx, p.n_act + n0, ti.e);
            } else {
              tma_load_3d(b_dst, &tmB, fb, kx, b_row, ti.e);
            }
          }
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
      if (CG == 2 && ok) {
        // the first CTA's MMA commits arrive on this CTA's empty barriers:
        // wait for the last one of every stage before the CTA may exit
        for (int s = 0; s < STAGES && ok; ++s) {
          ok = mbar_wait(bar_empty + 8 * stage, phase ^ 1, s_abort, &g_err_gemm,
                         kErrProducerTimeout);
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
      if (!ok && (CG == 1 || rank == 0)) {
        // drain: never exit with TMA writes into this CTA's smem in flight
        // (a pair's second CTA counts its copies on the first CTA's
        // barriers, which the first CTA drains for both)
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
          if (issued[s])
            mbar_wait(bar_full + 8 * s, issued_phase[s], &no_abort, &g_err_gemm,
                      kErrDrainTimeout, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool ok = true;
      bool any = false;
      // a pair MMA frees the stage and fills the accumulator in both CTAs
      const uint32_t empty1 = CG == 2 ? mapa_shared(bar_empty, 1) : 0u;
      const uint32_t accf1 = CG == 2 ? mapa_shared(bar_accf, 1) : 0u;
      const uint32_t empty0 = CG == 2 ? mapa_shared(bar_empty, 0) : bar_empty;
      const uint32_t accf0 = CG == 2 ? mapa_shared(bar_accf, 0) : bar_accf;
      // The issuer needs no tile coordinates: it walks this CTA's quant
      // blocks in order (tiles tile0, +tstride, ...), one TMEM
      // accumulator buffer per block.  Shared memory filled by TMA is made
      // visible by the full-barrier wait itself; the tcgen05 fence is only
      // needed after the accumulator hand-back, which the epilogue's
      // tcgen05.ld precede.
      const int my_tiles = tile0 < total_tiles ? (total_tiles - 1 - tile0) / tstride + 1 : 0;
      const int n_blocks = my_tiles * p.nq;
      int qb = 0;
      for (int i = 0; i < n_blocks; ++i) {
        if (!mbar_wait(bar_acce + 8 * acc, aphase ^ 1, s_abort, &g_err_gemm, kErrMmaTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int kt0 = qb * p.ktpq;
        const int kt1 = min(kt0 + p.ktpq, p.kt_total);
        for (int kt = kt0; kt < kt1; ++kt) {
          if (!mbar_wait(bar_full + 8 * stage, phase, s_abort, &g_err_gemm, kErrMmaTimeout)) {
            ok = false;
            break;
          }
          const uint32_t a_addr = sbase + SmemLayout::kA + stage * kTileABytes;
          const uint32_t b_addr = sbase + SmemLayout::kB + stage * kTileBBytes;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t ad = sw128_kmajor_desc(a_addr + k * 32);
            const uint64_t bd = sw128_kmajor_desc(b_addr + k * 32);
            if constexpr (CG == 2)
              umma_i8_pair(d_tmem, ad, bd, kIdesc, (kt > kt0 || k > 0) ? 1u : 0u);
            else
              umma_i8(d_tmem, ad, bd, kIdesc, (kt > kt0 || k > 0) ? 1u : 0u);
          }
          any = true;
          if constexpr (CG == 2) {
            umma_commit_pair(empty0 + 8 * stage);
            umma_commit_pair(empty1 + 8 * stage);
          } else {
            umma_commit(bar_empty + 8 * stage);
          }
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        if constexpr (CG == 2) {
          umma_commit_pair(accf0 + 8 * acc);
          umma_commit_pair(accf1 + 8 * acc);
        } else {
          umma_commit(bar_accf + 8 * acc);
        }
        if (++acc == NACC) acc = 0, aphase ^= 1;
        if (++qb == p.nq) qb = 0;
      }
      // wait for every issued MMA before TMEM can be released
      if (any) {
        if constexpr (CG == 2)
          umma_commit_pair(mapa_shared(bar_final, 0));
        else
          umma_commit(bar_final);
        volatile int no_abort = 0;
        mbar_wait(bar_final, 0, &no_abort, &g_err_gemm, kErrDrainTimeout, 200000000ull);
      }
    }
    __syncwarp();
  }
  } else {
    // register split, epilogue warpgroups: take the registers given back
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(EP::kRegsHigh));
    // ================= epilogue (16 or 8 warps) =================
    // TMEM lane quadrant = warp % 4 (hardware rule), column group cq =
    // (warp - kEpiW0) / 4.  Each thread owns one row and kCols accumulator
    // columns:
    //   kEpiStore, 16 warps:   tile columns [64cq, 64cq+64), one 64-column
    //                          weight-scale block, one Q_A * Q_B factor;
    //   kEpiStore, 8 wide warps (one CTA per tile): tile columns
    //                          [128cq, +128), two weight-scale blocks with
    //                          one factor each (the second in the "up" slot);
    //   kEpiSiluQuant:         gate columns [32cq, +32) and the matching up
    //                          columns [128+32cq, +32): one factor for each.
    // Four (two) warps share each SM sub-partition, which keeps the integer
    // multiply-add pipe busy while the other warps wait for their TMEM loads.
    const int quad = warp & 3;
    const int cq = (warp - kEpiW0) >> 2;
    const uint32_t t_lane = static_cast<uint32_t>(quad * 32) << 16;
    constexpr bool kFused = EPI == kEpiSiluQuant;
    constexpr bool kTwoQ = kFused || kWide;  // a second weight-scale factor per block
    auto chunk_col = [&](int c) -> uint32_t {  // TMEM column of 16-column chunk c
      if (kFused) return (c < 2) ? 32 * cq + 16 * c : 128 + 32 * cq + 16 * (c - 2);
      return EP::kCols * cq + 16 * c;
    };
    // first output column of this thread in tile t (w13 gate column when fused)
    auto first_col = [&](const TileInfo& u) -> int {
      return kFused ? u.nt * 128 + (EP::kCols / 2) * cq : u.nt * BN + EP::kCols * cq;
    };
    // the column of the second weight-scale factor's block: the up column
    // (fused), or the second 64 columns (wide); -1 past the output
    auto second_col = [&](int col) -> int {
      if (kFused) return p.n_act + col;
      return col + 64 < p.N ? col + 64 : -1;
    };
    auto col_valid = [&](int col) -> bool { return col < (kFused ? p.n_act : p.N); };
    int acc = 0;
    uint32_t aphase = 0;
    bool ok = true;
    // Every lane of a warp shares one scale row (a 32-row group never
    // straddles a tile_m boundary) and one weight-scale block per column
    // half, so the factor Q_A * Q_B of a quant block is warp-uniform: lane l
    // holds that of block (qb0 + l), and each block's factor is broadcast by
    // shuffle.  The next tile's Q factors and this tile's F factors travel by
    // cp.async into per-thread shared-memory slots while the accumulation
    // runs, so they take no registers from the accumulator.
    // Slots: [Q_A, Q_B, Q_B(up)] for even local tiles, the same for odd
    // ones, then F_A, F_B, F_B(up); a slot set is refilled only for the tile
    // after next, so an asynchronous write never meets a pending read.
    const uint32_t s_slot = sbase + SmemLayout::kSlots + 4 * (threadIdx.x - 32 * kEpiW0);
    constexpr uint32_t kSA = SmemLayout::kSlotArray;
    const uint32_t s_fa = s_slot + 6 * kSA;
    const uint32_t s_fb = s_slot + 7 * kSA;
    const uint32_t s_fbu = s_slot + 8 * kSA;
    auto ld_s32 = [](uint32_t a) {
      int v;
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
      return v;
    };
    auto st_s32 = [](uint32_t a, int v) {
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
    };
    // Q_A * Q_B of quant block (qb0 + lane) of tile t, synchronously (only
    // for more than 32 quant blocks); `second` selects the second factor
    auto tile_q = [&](int t, int qb0, bool second) -> int {
      const TileInfo u = decode_tile_cta<CG>(t, mt_prefix, p.E, p.n_tiles, rank);
      const int wrow = u.mt * BM + quad * 32;
      const int col = first_col(u);
      const int qb = qb0 + lane;
      if (MODE != kHybrid || wrow >= m_rows[u.e] || !col_valid(col) || qb >= p.nq) return 0;
      const int srow = so_prefix[u.e] + wrow / p.tile_m;
      const int c2 = second ? second_col(col) : col;
      if (c2 < 0) return 0;
      const int jb = c2 / 64;
      return __ldg(p.qa + static_cast<int64_t>(srow) * p.q_stride + qb) *
             __ldg(p.qb + (static_cast<int64_t>(u.e) * p.nsb + jb) * p.q_stride + qb);
    };
    // Q_A / Q_B (/ Q_B of the up half) of quant blocks 0..31 (one per lane)
    // of tile t, into slot set `par` asynchronously
    auto fetch_q = [&](int t, int par) {
      const uint32_t s_qa = s_slot + (3 * par) * kSA, s_qb = s_qa + kSA, s_qbu = s_qb + kSA;
      bool any = false;
      if (MODE == kHybrid && t < total_tiles) {
        const TileInfo u = decode_tile_cta<CG>(t, mt_prefix, p.E, p.n_tiles, rank);
        const int wrow = u.mt * BM + quad * 32;
        const int col = first_col(u);
        const int qb = lane;
        if (wrow < m_rows[u.e] && col_valid(col) && qb < p.nq) {
          const int srow = so_prefix[u.e] + wrow / p.tile_m;
          const int32_t* qb_e = p.qb + static_cast<int64_t>(u.e) * p.nsb * p.q_stride + qb;
          cp_async4(s_qa, p.qa + static_cast<int64_t>(srow) * p.q_stride + qb);
          cp_async4(s_qb, qb_e + static_cast<int64_t>(col / 64) * p.q_stride);
          if (kTwoQ) {
            const int c2 = second_col(col);
            if (c2 >= 0)
              cp_async4(s_qbu, qb_e + static_cast<int64_t>(c2 / 64) * p.q_stride);
            else
              st_s32(s_qbu, 0);
          }
          any = true;
        }
      }
      if (!any) {
        st_s32(s_qa, 0);
        st_s32(s_qb, 0);
        if (kTwoQ) st_s32(s_qbu, 0);
      }
    };
    fetch_q(tile0, 0);
    int par = 0;
    int lt = 0;  // fused epilogues run so far (absmax barrier phase and slots)
    for (int t = tile0; t < total_tiles && ok; t += tstride, par ^= 1) {
      cp_async_wait_all();
      int qv, qvu = 0;
      {
        const uint32_t s_qa = s_slot + (3 * par) * kSA;
        const int qa = ld_s32(s_qa);
        qv = qa * ld_s32(s_qa + kSA);
        if (kTwoQ) qvu = qa * ld_s32(s_qa + 2 * kSA);
      }
      fetch_q(t + tstride, par ^ 1);
      // CG == 2: this CTA's half of the pair tile may lie past the expert's
      // rows; its accumulator is then released unread and nothing is stored
      const TileInfo tc = decode_tile_cta<CG>(t, mt_prefix, p.E, p.n_tiles, rank);
      const bool own_ok = CG == 1 || tc.mt * BM < m_rows[tc.e];
      {
        // F_A, F_B (, F_B of the up half) of this tile, for the output phase
        const TileInfo& ti = tc;
        const int wrow0 = ti.mt * BM + quad * 32;
        const int col0 = first_col(ti);
        if (MODE == kHybrid && wrow0 < m_rows[ti.e] && col_valid(col0)) {
          const int srow = so_prefix[ti.e] + wrow0 / p.tile_m;
          const float* fb_e = p.fb + static_cast<int64_t>(ti.e) * p.nsb * p.f_stride;
          cp_async4(s_fa, p.fa + static_cast<int64_t>(srow) * p.f_stride);
          cp_async4(s_fb, fb_e + static_cast<int64_t>(col0 / 64) * p.f_stride);
          if (kTwoQ) {
            const int c2 = second_col(col0);
            if (c2 >= 0) cp_async4(s_fbu, fb_e + static_cast<int64_t>(c2 / 64) * p.f_stride);
          }
        }
      }
      int32_t W[EP::kCols];
      // The store epilogue writes its sums with the first quant block
      // (W = q * P) and takes its chunks through asm blocks (tmem_mad16 /
      // tmem_mul16, or the 32-column forms for the wide warps) whose loaded
      // values never become C variables: that keeps the sums in registers
      // without spills.  The fused SiLU epilogue keeps the plain form, which
      // spills less there.
      if (kFused || p.nq == 0) {
#pragma unroll
        for (int i = 0; i < EP::kCols; ++i) W[i] = 0;
      }
      // One 16-column chunk in flight per warp: with four epilogue warps on
      // each SM sub-partition the other warps' multiply-adds cover the TMEM
      // load latency (two chunks in flight measured slower: the second
      // buffer's registers cost spills).  The accumulator buffer goes back to
      // the MMA warp as soon as its last chunk has landed.
      uint32_t P[16];
      for (int qb = 0; qb < p.nq && ok; ++qb) {
        const int q = __shfl_sync(0xffffffffu, qv, qb & 31);
        const int qu = kTwoQ ? __shfl_sync(0xffffffffu, qvu, qb & 31) : 0;
        if ((qb & 31) == 31 && qb + 1 < p.nq) {  // K > 4096: the next 32 factors
          qv = tile_q(t, qb + 1, false);
          if (kTwoQ) qvu = tile_q(t, qb + 1, true);
        }
        if (!mbar_wait(bar_accf + 8 * acc, aphase, s_abort, &g_err_gemm, kErrEpilogueTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (!own_ok) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acce0 + 8 * acc);
          if (++acc == NACC) acc = 0, aphase ^= 1;
          continue;
        }
        if constexpr (kWide) {
          // four 32-column chunks of tile columns [128cq, +128), q for the
          // first 64 columns, qu for the other 64.  Each chunk is one asm
          // block (load, wait, 32 multiply-adds) whose
          // loaded values never become C variables; the last one hands the
          // accumulator back as soon as its load has landed (every thread
          // arrives).  Double-buffering the loads through C arrays measured
          // slower (w2 206 against 190 us).
          const uint32_t tb0 = tmem_base + t_lane + acc * BN + 128 * cq;
          const uint32_t tb1 = tb0 + 64;
          const uint32_t rb = bar_acce + 8 * acc;
          const int q0 = MODE == kHybrid ? q : 1;
          const int q1 = MODE == kHybrid ? qu : 1;
          if (qb == 0) {
            tmem_mul32(tb0, q0, 0u, W);
            tmem_mul32(tb0 + 32, q0, 0u, W + 32);
            tmem_mul32(tb1, q1, 0u, W + 64);
            tmem_mul32_release(tb1 + 32, q1, rb, W + 96);
          } else {
            tmem_mad32(tb0, q0, 0u, W);
            tmem_mad32(tb0 + 32, q0, 0u, W + 32);
            tmem_mad32(tb1, q1, 0u, W + 64);
            tmem_mad32_release(tb1 + 32, q1, rb, W + 96);
          }
          if (++acc == NACC) acc = 0, aphase ^= 1;
        } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if constexpr (!kFused) {
            if (c < 3) {
              const int qc = MODE == kHybrid ? q : 1;
              const uint32_t ta = tmem_base + t_lane + acc * BN + chunk_col(c);
#define I8_W16(b) W[b], W[b + 1], W[b + 2], W[b + 3], W[b + 4], W[b + 5], W[b + 6], W[b + 7], \
    W[b + 8], W[b + 9], W[b + 10], W[b + 11], W[b + 12], W[b + 13], W[b + 14], W[b + 15]
              if (qb == 0)
                tmem_mul16(ta, qc, I8_W16(16 * c));
              else
                tmem_mad16(ta, qc, I8_W16(16 * c));
#undef I8_W16
              continue;
            }
          }
          tmem_ld16(tmem_base + t_lane + acc * BN + chunk_col(c), P);
          tmem_wait_ld(P);
          if (c == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (CG == 2)
                mbar_arrive_cluster(acce0 + 8 * acc);
              else
                mbar_arrive(bar_acce + 8 * acc);
            }
            if (++acc == NACC) acc = 0, aphase ^= 1;
          }
          if (!kFused && qb == 0) {
            const int qc = MODE == kHybrid ? q : 1;
#pragma unroll
            for (int i = 0; i < 16; ++i) W[16 * c + i] = qc * static_cast<int32_t>(P[i]);
          } else if (MODE == kHybrid) {
            const int qc = (kFused && c >= 2) ? qu : q;
#pragma unroll
            for (int i = 0; i < 16; ++i) W[16 * c + i] += qc * static_cast<int32_t>(P[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) W[16 * c + i] += static_cast<int32_t>(P[i]);
          }
        }
        }  // narrow epilogue
      }
      if (!ok) break;
      if (!own_ok) continue;
      const TileInfo& ti = tc;
      const int m_e = m_rows[ti.e];
      const int wrow0 = ti.mt * BM + quad * 32;
      const int lrow = wrow0 + lane;
      const int col0 = first_col(ti);
      if constexpr (kFused) {
        // ---- SiLU(gate) * up + INT8 requant of the intermediate ----
        // mm1 = dtype(float(W) * (F_A * F_B)) (+ bias) exactly as the store
        // epilogue would write it; then act = dtype(dtype(silu(g)) * up) and
        // the quant of the (tile_m rows x 128 columns) block, with the same
        // element routines as the standalone fused SiLU-quant kernel.
        cp_async_wait_all();
        const float fa = __int_as_float(ld_s32(s_fa));
        const float fg = fa * __int_as_float(ld_s32(s_fb));
        const float fu = fa * __int_as_float(ld_s32(s_fbu));
        const bool row_ok = lrow < m_e;
        const float* bg = HAS_BIAS ? p.bias + static_cast<int64_t>(ti.e) * p.bias_stride + col0
                                   : nullptr;
        // kAC chunks of 8 activations: the thread's gate columns are W[0, kU)
        // and the matching up columns W[kU, 2 kU)
        constexpr int kU = EP::kCols / 2;
        constexpr int kAC = kU / 8;
        uint4 act[kAC];
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < kAC; ++j) {
          uint32_t g4[4], u4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = 8 * j + 2 * i;
            if (HAS_BIAS) {
              g4[i] = pack2<OutT>(bias_epi(W[c], fg, __ldg(bg + c)),
                                  bias_epi(W[c + 1], fg, __ldg(bg + c + 1)));
              u4[i] = pack2<OutT>(bias_epi(W[kU + c], fu, __ldg(bg + p.n_act + c)),
                                  bias_epi(W[kU + c + 1], fu, __ldg(bg + p.n_act + c + 1)));
            } else {
              g4[i] = pack2<OutT>(__fmul_rn(static_cast<float>(W[c]), fg),
                                  __fmul_rn(static_cast<float>(W[c + 1]), fg));
              u4[i] = pack2<OutT>(__fmul_rn(static_cast<float>(W[kU + c]), fu),
                                  __fmul_rn(static_cast<float>(W[kU + c + 1]), fu));
            }
          }
          uint4 a = silu_mul_chunk<OutT>(make_uint4(g4[0], g4[1], g4[2], g4[3]),
                                         make_uint4(u4[0], u4[1], u4[2], u4[3]));
          // rows of the next expert and columns past the intermediate size
          // take no part in the block absmax (n_act is a multiple of 8)
          if (!row_ok || !(col0 + 8 * j < p.n_act)) a = make_uint4(0u, 0u, 0u, 0u);
          m = fmaxf(m, chunk_absmax<OutT>(a));
          act[j] = a;
        }
        // block absmax over the tile_m rows: warp max, then a shared atomic
        // max per row group completed by a bounded mbarrier wait (no named
        // barrier, so a warp that gives up cannot leave the others blocked)
        const int grp = p.tile_m == 64 ? (quad >> 1) : 0;
        const int slot3 = lt % 3;
        unsigned* red = reinterpret_cast<unsigned*>(smem + SmemLayout::kRed) + 3 * grp;
        const unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
        if (lane == 0) {
          atomicMax(red + slot3, mb);
          mbar_arrive(bar_red + 8 * grp);
        }
        if (!mbar_wait(bar_red + 8 * grp, static_cast<uint32_t>(lt & 1), s_abort, &g_err_gemm,
                       kErrEpilogueTimeout)) {
          ok = false;
          break;
        }
        const float amax = __uint_as_float(*reinterpret_cast<volatile unsigned*>(red + slot3));
        // the group's first warp clears the slot of the tile after next: every
        // warp of the group has read it (it was this tile's previous use)
        const bool lead = cq == 0 && quad == (p.tile_m == 64 ? 2 * grp : 0) && lane == 0;
        if (lead) red[(lt + 2) % 3] = 0u;
        const float scale = __fdiv_rn(fmaxf(amax, 1e-10f), 127.0f);
        const QuantInv qi = quant_inv(scale);
        const int grow0 = ti.mt * BM + (p.tile_m == 64 ? 64 * grp : 0);
        if (lead && grow0 < m_e) {
          const int srow = so_prefix[ti.e] + grow0 / p.tile_m;
          p.act_scale[static_cast<int64_t>(srow) * p.kb_act + ti.nt] = scale;
        }
        uint32_t qw[2 * kAC];
#pragma unroll
        for (int j = 0; j < kAC; ++j) {
          uint2 q2;
          if (!quant_chunk_bracket<OutT>(act[j], qi, q2)) q2 = quant_chunk_exact16<OutT>(act[j], scale);
          qw[2 * j] = q2.x;
          qw[2 * j + 1] = q2.y;
        }
        if (wrow0 + 32 <= m_e && col0 + kU <= p.n_act) {
          // whole warp inside the expert: 32 rows x 32 bytes per TMA tensor
          // store (kU / 32 of them), staged with the 32-byte swizzle
          const uint32_t stg = sbase + SmemLayout::kStg + (warp - kEpiW0) * SmemLayout::kStgWarpBytes;
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
#pragma unroll
          for (int s32 = 0; s32 < kU / 32; ++s32) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t a = stg + 1024 * s32 + 32 * lane + 16 * (h ^ ((lane >> 2) & 1));
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                           "r"(qw[8 * s32 + 4 * h]), "r"(qw[8 * s32 + 4 * h + 1]),
                           "r"(qw[8 * s32 + 4 * h + 2]), "r"(qw[8 * s32 + 4 * h + 3])
                           : "memory");
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int s32 = 0; s32 < kU / 32; ++s32)
              tma_store_2d(&tmO, stg + 1024 * s32, col0 + 32 * s32, e_row0[ti.e] + wrow0);
            bulk_commit();
          }
        } else if (row_ok) {
          int8_t* dst = p.act_q + static_cast<int64_t>(e_row0[ti.e] + lrow) * p.n_act + col0;
#pragma unroll
          for (int j = 0; j < kAC; ++j)
            if (col0 + 8 * j < p.n_act)
              *reinterpret_cast<uint2*>(dst + 8 * j) = make_uint2(qw[2 * j], qw[2 * j + 1]);
        }
        ++lt;
        continue;
      }
      // ---- convert, scale, round, store (per 64-column half) ----
      constexpr int kHalves = EP::kCols / 64;
      float fh[kHalves];
      if (MODE == kHybrid) {
        cp_async_wait_all();
        const float fa = __int_as_float(ld_s32(s_fa));
        fh[0] = fa * __int_as_float(ld_s32(s_fb));
        if constexpr (kHalves == 2) fh[1] = fa * __int_as_float(ld_s32(s_fbu));
      } else {
        const float f = p.a_row_scale == nullptr
                            ? p.alpha
                            : (lrow < m_e ? __ldg(p.a_row_scale + e_row0[ti.e] + lrow) *
                                                __ldg(p.b_expert_scale + ti.e)
                                          : 0.f);
#pragma unroll
        for (int hh = 0; hh < kHalves; ++hh) fh[hh] = f;
      }
#pragma unroll
      for (int hh = 0; hh < kHalves; ++hh) {
        const float f = fh[hh];
        const int colh = col0 + 64 * hh;
        const int32_t* Wh = W + 64 * hh;
        if constexpr (!std::is_same<OutT, int32_t>::value) {
          if (wrow0 + 32 <= m_e && colh + 64 <= p.N) {
            // All 32 rows belong to this expert: stage the warp's 32 x 64
            // block in shared memory (64-byte swizzle, conflict-free) and
            // write it with two TMA tensor stores of 32 x 32, so the stores
            // leave as whole lines instead of 32 row fragments per
            // instruction.  Wide warps alternate two staging buffers.
            const uint32_t stg = sbase + SmemLayout::kStg +
                                 (warp - kEpiW0) * SmemLayout::kStgWarpBytes +
                                 hh * SmemLayout::kStgBufBytes;
            const float* bp =
                HAS_BIAS ? p.bias + static_cast<int64_t>(ti.e) * p.bias_stride + colh : nullptr;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              // the previous store from this buffer has read it (wide: the
              // other buffer's latest store may still be reading)
              if (lane == 0) {
                if (kWide && h == 0)
                  bulk_wait_read1();
                else
                  bulk_wait_read0();
              }
              __syncwarp();
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint32_t w4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const int c = 32 * h + 8 * j + 2 * i;
                  if (HAS_BIAS) {
                    w4[i] = pack2<OutT>(bias_epi(Wh[c], f, __ldg(bp + c)),
                                        bias_epi(Wh[c + 1], f, __ldg(bp + c + 1)));
                  } else {
                    w4[i] = pack2<OutT>(__fmul_rn(static_cast<float>(Wh[c]), f),
                                        __fmul_rn(static_cast<float>(Wh[c + 1]), f));
                  }
                }
                const uint32_t a = stg + 64 * lane + 16 * (j ^ ((lane >> 1) & 3));
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w4[0]),
                             "r"(w4[1]), "r"(w4[2]), "r"(w4[3])
                             : "memory");
              }
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmO, stg, colh + 32 * h, e_row0[ti.e] + wrow0);
                bulk_commit();
              }
            }
            continue;
          }
        }
        if (!(lrow < m_e && colh < p.N)) continue;
        const int64_t row_off = static_cast<int64_t>(e_row0[ti.e] + lrow) * p.N + colh;
        const int ncols = min(64, p.N - colh);
        if constexpr (std::is_same<OutT, int32_t>::value) {
          // raw accumulator output (verification mode)
          int32_t* dst = static_cast<int32_t*>(p.out) + row_off;
          (void)f;
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (4 * c < ncols)
              *reinterpret_cast<int4*>(dst + 4 * c) =
                  make_int4(Wh[4 * c], Wh[4 * c + 1], Wh[4 * c + 2], Wh[4 * c + 3]);
        } else {
          OutT* dst = static_cast<OutT*>(p.out) + row_off;
          const float* bp =
              HAS_BIAS ? p.bias + static_cast<int64_t>(ti.e) * p.bias_stride + colh : nullptr;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            if (8 * c >= ncols) continue;
            uint32_t w4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int j = 8 * c + 2 * i;
              if (HAS_BIAS) {
                w4[i] = pack2<OutT>(bias_epi(Wh[j], f, __ldg(bp + j)),
                                    bias_epi(Wh[j + 1], f, __ldg(bp + j + 1)));
              } else {
                w4[i] = pack2<OutT>(__fmul_rn(static_cast<float>(Wh[j]), f),
                                    __fmul_rn(static_cast<float>(Wh[j + 1]), f));
              }
            }
            *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
      }
    }
    cp_async_wait_all();  // no asynchronous copy into shared memory outlives the CTA
    if (lane == 0) bulk_wait0();  // nor a tensor store still reading the staging buffer
  }

  tc_fence_before();
  __syncthreads();
  // neither CTA of a pair leaves while the other may still signal its
  // barriers or the pair MMA may still read its shared memory
  if constexpr (CG == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
int g_encode_status = I8MOE_OK;

int get_encode() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                     cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
      g_encode_status = I8MOE_ERR_CUDA;
    } else {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (g_encode_status != I8MOE_OK)
    return set_error(I8MOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  return I8MOE_OK;
}

int make_tmap_a(CUtensorMap* m, const int8_t* a, int64_t rows, int64_t k) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k)};
  cuuint32_t box[2] = {BK, BM};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(a), dims, strides,
                        box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(I8MOE_ERR_CUDA, "cuTensorMapEncodeTiled(A) failed");
  return I8MOE_OK;
}

// B box: all BN rows of the tile, or (fused SiLU epilogue) the 128 gate and
// the 128 up rows as two loads
int make_tmap_b(CUtensorMap* m, const int8_t* b, int64_t E, int64_t n, int64_t k, int box_rows) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(n),
                        static_cast<cuuint64_t>(E)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(n * k)};
  cuuint32_t box[3] = {BK, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(b), dims, strides,
                        box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(I8MOE_ERR_CUDA, "cuTensorMapEncodeTiled(B) failed");
  return I8MOE_OK;
}

int make_tmap_out(CUtensorMap* m, void* out, int out_dtype, int64_t rows, int64_t n) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(n * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  const CUtensorMapDataType dt = out_dtype == I8MOE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = g_encode(m, dt, 2, out, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(I8MOE_ERR_CUDA, "cuTensorMapEncodeTiled(out) failed");
  return I8MOE_OK;
}

// int8 activation output of the fused SiLU epilogue: boxes of 32 x 32 bytes
int make_tmap_act(CUtensorMap* m, int8_t* act, int64_t rows, int64_t n_act) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(n_act), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(n_act)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, act, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(I8MOE_ERR_CUDA, "cuTensorMapEncodeTiled(act) failed");
  return I8MOE_OK;
}

// Launches one instantiation persistently: one CTA per SM (CG == 1) or as
// many CTA pairs as can be resident at once (CG == 2, clusters of two), never
// more than there are tiles.
template <int MODE, bool HAS_BIAS, typename OutT, int EPI, int CG>
int launch_cg(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
              const GemmParams& p, int64_t upper_tiles, cudaStream_t st) {
  auto kern = grouped_gemm_kernel<MODE, HAS_BIAS, OutT, EPI, CG>;
  using EP = Epi<EPI, CG>;
  const int smem = SmemLayout<CG, EPI>::bytes(p.E) + 1024;
  const int smem_max = std::min(SmemLayout<CG, EPI>::bytes(kMaxExperts) + 1024, kSmemLimit);
  if (smem > smem_max) return set_error(I8MOE_ERR_UNSUPPORTED, "grouped GEMM: too many experts");
  static int attr_done[64] = {0};
  static int max_clusters[64] = {0};
  const int dev = current_device();
  const bool cached = dev >= 0 && dev < 64 && __atomic_load_n(&attr_done[dev], __ATOMIC_ACQUIRE);
  int n_pairs = 0;
  if (!cached) {
    // the register split is exact: any other launch count would leave the
    // epilogue's setmaxnreg.inc waiting (fewer) or fail to launch (more)
    cudaFuncAttributes fa;
    I8_CUDA(cudaFuncGetAttributes(&fa, kern));
    I8_REQUIRE(fa.numRegs == EP::kRegsLaunch,
               "grouped GEMM: compiled with %d registers a thread; its register split needs %d",
               fa.numRegs, EP::kRegsLaunch);
    I8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
    if (CG == 2) {
      cudaLaunchConfig_t q = {};
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.gridDim = dim3(2 * static_cast<unsigned>(num_sms(dev) / 2));
      q.blockDim = dim3(EP::kThreads);
      q.dynamicSmemBytes = smem_max;
      q.attrs = qa;
      q.numAttrs = 1;
      I8_CUDA(cudaOccupancyMaxActiveClusters(&n_pairs, kern, &q));
      if (n_pairs < 1) return set_error(I8MOE_ERR_UNSUPPORTED, "no CTA pair fits on the device");
    }
    if (dev >= 0 && dev < 64) {
      __atomic_store_n(&max_clusters[dev], n_pairs, __ATOMIC_RELAXED);
      __atomic_store_n(&attr_done[dev], 1, __ATOMIC_RELEASE);
    }
  } else {
    n_pairs = __atomic_load_n(&max_clusters[dev], __ATOMIC_RELAXED);
  }
  if constexpr (CG == 2) {
    const int pairs = static_cast<int>(std::min<int64_t>(n_pairs, std::max<int64_t>(upper_tiles, 1)));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * static_cast<unsigned>(pairs));
    cfg.blockDim = dim3(EP::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    I8_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, to, p));
  } else {
    const int grid = static_cast<int>(std::min<int64_t>(num_sms(dev), std::max<int64_t>(upper_tiles, 1)));
    kern<<<grid, EP::kThreads, smem, st>>>(ta, tb, to, p);
  }
  return check_launch("grouped_gemm_kernel");
}

// CTA pairs: -1 chooses by problem shape, 0 never, 1 always (hybrid GEMMs).
int g_cta_pairs = -1;

// the pair layout's five-stage ring leaves room for the per-expert tables
// of up to ~700 experts within the 227 KB a CTA may use
bool pairs_fit(int64_t E) {
  return SmemLayout<2, kEpiStore>::bytes(static_cast<int>(E)) + 1024 <= kSmemLimit &&
         SmemLayout<2, kEpiSiluQuant>::bytes(static_cast<int>(E)) + 1024 <= kSmemLimit;
}

// Pair tiles cover 256 rows of one expert, so an expert with an odd number
// of 128-row m-tiles leaves half of its last pair tile idle.  Measured on
// B200 at the benchmark shapes, a pair tile's quant block takes as long as a
// single CTA's (~1.2-1.3 k cycles: the epilogue's instruction issue, not the
// 48 KB operand stream, bounds it), so the idle halves make pairs slower;
// the default (-1) is therefore one CTA per tile, and pairs are opt-in.
bool use_cta_pairs(int mode, int64_t sum_m, int64_t E) {
  (void)sum_m;
  if (mode != kHybrid || !pairs_fit(E)) return false;
  return __atomic_load_n(&g_cta_pairs, __ATOMIC_RELAXED) == 1;
}

template <int MODE, bool HAS_BIAS, typename OutT, int EPI = kEpiStore>
int launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
             const GemmParams& p, int64_t upper_tiles, bool pairs, cudaStream_t st) {
  if constexpr (MODE == kHybrid) {
    if (pairs) return launch_cg<MODE, HAS_BIAS, OutT, EPI, 2>(ta, tb, to, p, upper_tiles, st);
  }
  return launch_cg<MODE, HAS_BIAS, OutT, EPI, 1>(ta, tb, to, p, upper_tiles, st);
}

int check_device() {
  const int dev = current_device();
  int major = 0, minor = 0;
  I8_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  I8_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
  if (major != 10 || minor != 0)
    return set_error(I8MOE_ERR_UNSUPPORTED, "libi8moe GEMMs require an sm_100 (B200) device");
  return I8MOE_OK;
}

// epi == kEpiSiluQuant: `n` is the w13 output width 2*p.n_act, `out_dtype`
// the storage type of the intermediate (bf16/fp16), p.act_q / p.act_scale
// the outputs.
int launch_gemm(int mode, int out_dtype, bool has_bias, const int8_t* a, const int8_t* b,
                GemmParams p, int64_t E, int64_t sum_m, int64_t n, int64_t k, cudaStream_t st,
                int epi = kEpiStore) {
  I8_REQUIRE(out_dtype == I8MOE_BF16 || out_dtype == I8MOE_FP16 || out_dtype == I8MOE_S32,
             "out must be bfloat16 (or float16, or int32 for the raw accumulator)");
  if (epi == kEpiSiluQuant) {
    I8_REQUIRE(mode == kHybrid && out_dtype != I8MOE_S32, "fused SiLU epilogue: hybrid bf16/fp16 only");
    I8_REQUIRE(n == 2 * int64_t(p.n_act) && p.n_act % 32 == 0,
               "fused SiLU epilogue: the intermediate size must be a multiple of 32");
    I8_REQUIRE(p.act_q != nullptr && p.act_scale != nullptr && p.so != nullptr,
               "fused SiLU epilogue: act_q, act_scale and scale_offsets are required");
    I8_REQUIRE(reinterpret_cast<uintptr_t>(p.act_q) % 16 == 0, "act_q must be 16-byte aligned");
    p.out = p.act_q;  // for the alignment check below
  }
  I8_REQUIRE(E >= 1 && E <= kMaxExperts, "number of experts must be in [1, %d]", kMaxExperts);
  I8_REQUIRE(k % 32 == 0, "K must be divisible by 32 for INT8 tensor ops");
  I8_REQUIRE(n % 8 == 0, "N must be a multiple of 8 (16-byte output rows)");
  I8_REQUIRE(sum_m >= 0 && sum_m < (int64_t(1) << 31) && n > 0 && n < (int64_t(1) << 31) &&
                 k > 0 && k < (int64_t(1) << 31),
             "grouped GEMM: unsupported shape");
  I8_REQUIRE((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
              reinterpret_cast<uintptr_t>(p.out)) % 16 == 0,
             "grouped GEMM: a, b and out must be 16-byte aligned");
  if (sum_m == 0) return I8MOE_OK;
  int rc = check_device();
  if (rc) return rc;
  rc = get_encode();
  if (rc) return rc;
  const bool pairs = use_cta_pairs(mode, sum_m, E);
  CUtensorMap ta, tb;
  rc = make_tmap_a(&ta, a, sum_m, k);
  if (rc) return rc;
  // B box: 128 rows per load (fused epilogue: gate and up separately; CTA
  // pairs: each CTA its half), else the whole 256-row tile
  rc = make_tmap_b(&tb, b, E, n, k, (epi == kEpiSiluQuant || pairs) ? 128 : BN);
  if (rc) return rc;
  CUtensorMap to = ta;  // the raw int32 output is written without a tensor map
  if (epi == kEpiSiluQuant) {
    rc = make_tmap_act(&to, p.act_q, sum_m, p.n_act);
    if (rc) return rc;
  } else if (out_dtype != I8MOE_S32) {
    rc = make_tmap_out(&to, p.out, out_dtype, sum_m, n);
    if (rc) return rc;
  }
  p.E = static_cast<int>(E);
  p.sum_m = static_cast<int>(sum_m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.kt_total = static_cast<int>((k + BK - 1) / BK);
  p.k_pad = p.kt_total * BK - p.K;
  p.n_tiles = epi == kEpiSiluQuant ? (p.n_act + 127) / 128 : static_cast<int>((n + BN - 1) / BN);
  const int64_t upper_tiles = ((sum_m + BM - 1) / BM + E) * p.n_tiles;
  const int64_t grid = upper_tiles;  // launches cap it at the resident CTAs (pairs)
  if (epi == kEpiSiluQuant) {
    if (out_dtype == I8MOE_BF16)
      return has_bias ? launch_t<kHybrid, true, __nv_bfloat16, kEpiSiluQuant>(ta, tb, to, p, grid, pairs, st)
                      : launch_t<kHybrid, false, __nv_bfloat16, kEpiSiluQuant>(ta, tb, to, p, grid, pairs, st);
    return has_bias ? launch_t<kHybrid, true, __half, kEpiSiluQuant>(ta, tb, to, p, grid, pairs, st)
                    : launch_t<kHybrid, false, __half, kEpiSiluQuant>(ta, tb, to, p, grid, pairs, st);
  }
  if (out_dtype == I8MOE_S32) {
    I8_REQUIRE(!has_bias, "the raw int32 accumulator output takes no bias");
    return mode == kHybrid ? launch_t<kHybrid, false, int32_t>(ta, tb, to, p, grid, pairs, st)
                           : launch_t<kPerTensor, false, int32_t>(ta, tb, to, p, grid, pairs, st);
  }
  if (mode == kHybrid) {
    if (out_dtype == I8MOE_BF16)
      return has_bias ? launch_t<kHybrid, true, __nv_bfloat16>(ta, tb, to, p, grid, pairs, st)
                      : launch_t<kHybrid, false, __nv_bfloat16>(ta, tb, to, p, grid, pairs, st);
    return has_bias ? launch_t<kHybrid, true, __half>(ta, tb, to, p, grid, pairs, st)
                    : launch_t<kHybrid, false, __half>(ta, tb, to, p, grid, pairs, st);
  }
  if (out_dtype == I8MOE_BF16) return launch_t<kPerTensor, false, __nv_bfloat16>(ta, tb, to, p, grid, pairs, st);
  return launch_t<kPerTensor, false, __half>(ta, tb, to, p, grid, pairs, st);
}

}  // namespace
}  // namespace i8moe

using namespace i8moe;

extern "C" {

int i8moe_hybrid_grouped_gemm(const int8_t* a_q, const int32_t* a_qscale, const float* a_fscale,
                              int64_t a_scale_rows, const int8_t* b_q, const int32_t* b_qscale,
                              const float* b_fscale, const int32_t* expert_offsets,
                              const int32_t* problem_sizes, const int32_t* scale_offsets,
                              const float* bias, int64_t bias_stride, void* out, int out_dtype,
                              int64_t n_expert, int64_t sum_m, int64_t n, int64_t k,
                              int64_t quant_block_size, int64_t super_group_size,
                              int64_t tile_m, i8moe_stream_t stream) {
  (void)a_scale_rows;
  I8_REQUIRE(quant_block_size > 0, "quant_block_size must be positive");
  I8_REQUIRE(super_group_size > 0, "super_group_size must be positive");
  I8_REQUIRE(quant_block_size % BK == 0, "quant_block_size must be divisible by the selected TileK");
  I8_REQUIRE(tile_m == 64 || tile_m == 128, "tile_m must be 64 or 128");
  I8_REQUIRE(bias_stride == 0 || bias_stride == n, "bias must have shape [N] or [E, N]");
  const int64_t nqb = (k + quant_block_size - 1) / quant_block_size;
  GemmParams p{};
  p.eo = expert_offsets;
  p.ps = problem_sizes;
  p.so = scale_offsets;
  p.qa = a_qscale;
  p.fa = a_fscale;
  p.qb = b_qscale;
  p.fb = b_fscale;
  p.bias = bias;
  p.bias_stride = static_cast<int>(bias_stride);
  p.out = out;
  p.ktpq = static_cast<int>(quant_block_size / BK);
  p.nq = static_cast<int>((((k + BK - 1) / BK) + p.ktpq - 1) / p.ktpq);
  p.q_stride = static_cast<int>(nqb);
  p.f_stride = static_cast<int>((nqb + super_group_size - 1) / super_group_size);
  p.nsb = static_cast<int>((n + 63) / 64);
  p.tile_m = static_cast<int>(tile_m);
  return launch_gemm(kHybrid, out_dtype, bias != nullptr, a_q, b_q, p, n_expert, sum_m, n, k,
                     static_cast<cudaStream_t>(stream));
}

int i8moe_hybrid_grouped_gemm_silu_quant(
    const int8_t* a_q, const int32_t* a_qscale, const float* a_fscale, int64_t a_scale_rows,
    const int8_t* w13_q, const int32_t* w13_qscale, const float* w13_fscale,
    const int32_t* expert_offsets, const int32_t* problem_sizes, const int32_t* scale_offsets,
    const float* bias, int64_t bias_stride, int act_dtype, int64_t n_expert, int64_t sum_m,
    int64_t n_act, int64_t k, int64_t quant_block_size, int64_t super_group_size,
    int64_t tile_m, int64_t q_max, int8_t* act_q, int32_t* act_qscale, float* act_fscale,
    i8moe_stream_t stream) {
  (void)a_scale_rows;
  I8_REQUIRE(quant_block_size > 0 && quant_block_size % BK == 0,
             "quant_block_size must be a positive multiple of the selected TileK");
  I8_REQUIRE(super_group_size > 0 && q_max > 0, "super_group_size and q_max must be positive");
  I8_REQUIRE(tile_m == 64 || tile_m == 128, "tile_m must be 64 or 128");
  I8_REQUIRE(n_act > 0, "intermediate size must be positive");
  I8_REQUIRE(bias_stride == 0 || bias_stride == 2 * n_act, "bias must have shape [2N] or [E, 2N]");
  I8_REQUIRE(act_qscale != nullptr && act_fscale != nullptr, "act Q/F buffers are required");
  const int64_t nqb = (k + quant_block_size - 1) / quant_block_size;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmParams p{};
  p.eo = expert_offsets;
  p.ps = problem_sizes;
  p.so = scale_offsets;
  p.qa = a_qscale;
  p.fa = a_fscale;
  p.qb = w13_qscale;
  p.fb = w13_fscale;
  p.bias = bias;
  p.bias_stride = static_cast<int>(bias_stride);
  p.ktpq = static_cast<int>(quant_block_size / BK);
  p.nq = static_cast<int>((((k + BK - 1) / BK) + p.ktpq - 1) / p.ktpq);
  p.q_stride = static_cast<int>(nqb);
  p.f_stride = static_cast<int>((nqb + super_group_size - 1) / super_group_size);
  p.nsb = static_cast<int>((2 * n_act + 63) / 64);
  p.tile_m = static_cast<int>(tile_m);
  p.n_act = static_cast<int>(n_act);
  p.act_q = act_q;
  p.act_scale = reinterpret_cast<float*>(act_qscale);  // raw scales, factorised below
  p.kb_act = static_cast<int>((n_act + 127) / 128);
  int rc = launch_gemm(kHybrid, act_dtype, bias != nullptr, a_q, w13_q, p, n_expert, sum_m,
                       2 * n_act, k, st, kEpiSiluQuant);
  if (rc) return rc;
  if (sum_m == 0) return I8MOE_OK;
  const int64_t rows_upper = (sum_m + tile_m - 1) / tile_m + n_expert;
  return launch_scales_to_qf(reinterpret_cast<const float*>(act_qscale), rows_upper,
                             scale_offsets + n_expert, p.kb_act, q_max, super_group_size,
                             act_qscale, act_fscale, st);
}

int i8moe_int8_grouped_mm(const int8_t* a, const int8_t* b, void* out, int out_dtype,
                          float alpha, const float* a_row_scale, const float* b_expert_scale,
                          const int32_t* expert_offsets, const int32_t* problem_sizes,
                          int64_t n_expert, int64_t sum_m, int64_t n, int64_t k,
                          i8moe_stream_t stream) {
  I8_REQUIRE((a_row_scale == nullptr) == (b_expert_scale == nullptr),
             "a_row_scale and b_expert_scale must be given together");
  GemmParams p{};
  p.eo = expert_offsets;
  p.ps = problem_sizes;
  p.alpha = alpha;
  p.a_row_scale = a_row_scale;
  p.b_expert_scale = b_expert_scale;
  p.out = out;
  const int64_t kt = (k + BK - 1) / BK;
  p.ktpq = static_cast<int>(kt);
  p.nq = 1;
  p.tile_m = BM;
  return launch_gemm(kPerTensor, out_dtype, false, a, b, p, n_expert, sum_m, n, k,
                     static_cast<cudaStream_t>(stream));
}

// Selects the CTA-pair GEMM variant: -1 by problem shape (default), 0 never,
// 1 always.  Returns the previous setting.
int i8moe_gemm_set_cta_pairs(int mode) {
  I8_REQUIRE(mode >= -1 && mode <= 1, "cta pairs: mode must be -1, 0 or 1");
  return __atomic_exchange_n(&g_cta_pairs, mode, __ATOMIC_RELAXED);
}

}  // extern "C"
