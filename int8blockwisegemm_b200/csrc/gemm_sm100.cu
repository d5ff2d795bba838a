// Persistent grouped INT8 GEMMs on the 5th-generation tensor cores (sm_100a).
//
// One kernel template serves
//   * the hybrid blockwise GEMM (reference
//     csrc/int8_hybrid_grouped_gemm.cu:218-479): for every 128-deep K-tile
//     (or quant block of several K-tiles) the int32 partial product is
//     multiplied by Q_A[s, qb] * Q_B[e, n/64, qb] and added to an int32
//     running sum; at the end out = dtype(float(W) * (F_A[s,0] * F_B[e,n/64,0]))
//     (+ bias via fma for the _bias variants);
//   * the per-tensor grouped GEMM (csrc/int8_grouped_gemm.cu:35-47,193-219):
//     out = dtype(float(sum_k a*b) * alpha) with alpha per tensor, or
//     per-token x per-expert (extension).
//
// Structure (one CTA per SM, 18 warps; tiles of 128 rows x 256 columns):
//   warp 0      TMA producer: A tile [128 rows x 128 K] and B tile
//               [BN x 128 K] per K-tile, 128-byte swizzle, into a STAGES-deep
//               shared-memory ring guarded by full/empty mbarriers.
//   warp 1      TMEM allocator + single-thread MMA issuer:
//               tcgen05.mma.cta_group::1.kind::i8, M=128, N=256, K=32, four
//               per K-tile, accumulating one quant block into one of two TMEM
//               accumulator buffers (256 columns each); tcgen05.commit frees
//               the smem stage and, at the end of a quant block, signals the
//               epilogue.
//   warps 2..17 epilogue: TMEM lane quadrant = warp % 4, column quarter =
//               (warp - 2) / 4.  Each thread owns one output row and 64
//               columns: tcgen05.ld the block partial in 16-column chunks
//               (other warps' accumulation covers each load's latency),
//               release the TMEM buffer, W += q * P (int32 IMAD); after the
//               last block convert, scale, round and store the row with 16-B
//               stores (rows beyond the expert are not stored, so
//               neighbouring experts are never overwritten).
//               The hybrid format costs one integer multiply-add per output
//               element per quant block, which at 128-deep blocks matches the
//               tensor-core rate; 16 warps keep that pipe fed.
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
constexpr int STAGES = 3;
constexpr int NACC = 2;
constexpr int kEpiWarps = 16;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer + MMA + epilogue warps
constexpr int kMaxExperts = 1024;
constexpr int kTileABytes = BM * BK;
constexpr int kTileBBytes = BN * BK;
constexpr uint32_t kTmemCols = NACC * BN;
constexpr uint32_t kIdesc = idesc_i8(BM, BN);

enum GemmMode { kHybrid = 0, kPerTensor = 1 };

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
  int prefetch;  // K-tiles prefetched into L2 ahead of the smem loads (0: off)
};

struct SmemLayout {
  static constexpr int kA = 0;
  static constexpr int kB = kA + STAGES * kTileABytes;
  // per-epilogue-warp output staging (32 rows x 64 B, 64-byte swizzle)
  static constexpr int kStg = kB + STAGES * kTileBBytes;  // 1024-B aligned
  static constexpr int kStgWarpBytes = 32 * 64;
  static constexpr int kBar = kStg + kEpiWarps * kStgWarpBytes;  // 8-B aligned
  static constexpr int kNumBars = 2 * STAGES + 2 * NACC + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;   // tmem base, abort flag
  // per-epilogue-thread slots (Q_A, Q_B per tile parity; F_A, F_B of the
  // current tile), then the per-expert tables: m-tile prefix, scale-row
  // offset, row count, first row
  static constexpr int kSlots = kMisc + 16;
  static constexpr int kSlotArray = 4 * 32 * kEpiWarps;
  static constexpr int kPrefix = kSlots + 6 * kSlotArray;
  static constexpr int bytes(int E) { return kPrefix + 4 * (E + 1) * 4 + 32; }
};

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

template <int MODE, bool HAS_BIAS, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO, const GemmParams p) {
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
  for (int e = threadIdx.x; e < p.E; e += kThreads) {
    const int m = max(0, __ldg(p.ps + 3 * e));
    mt_prefix[e] = (m + BM - 1) / BM;
    so_prefix[e] = p.so ? __ldg(p.so + e) : (m + p.tile_m - 1) / p.tile_m;
    m_rows[e] = m;
    e_row0[e] = __ldg(p.eo + e);
  }
  if (threadIdx.x == 0) *s_abort = 0;
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
      mbar_init(bar_acce + 8 * a, kEpiWarps);
    }
    mbar_init(bar_final, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

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
      // With p.prefetch > 0, the K-tile p.prefetch steps ahead of the one
      // being loaded into shared memory (possibly in the next tile) is
      // prefetched into L2 so first touches of weight tiles in HBM overlap.
      int t = blockIdx.x;
      TileInfo ti = decode_tile(t < total_tiles ? t : 0, mt_prefix, p.E, p.n_tiles);
      int row0 = e_row0[ti.e] + ti.mt * BM;
      int tn = t + gridDim.x;
      TileInfo tin = decode_tile(tn < total_tiles ? tn : 0, mt_prefix, p.E, p.n_tiles);
      int row0n = e_row0[tin.e] + tin.mt * BM;
      for (; t < total_tiles && ok; t += gridDim.x) {
        const int n0 = ti.nt * BN;
        for (int kt = 0; kt < p.kt_total; ++kt) {
          if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1, s_abort, &g_err_gemm,
                         kErrProducerTimeout)) {
            ok = false;
            break;
          }
          const int kx = kt * BK - p.k_pad;
          const uint32_t fb = bar_full + 8 * stage;
          mbar_arrive_expect_tx(fb, kTileABytes + kTileBBytes);
          tma_load_2d(sbase + SmemLayout::kA + stage * kTileABytes, &tmA, fb, kx, row0);
          tma_load_3d(sbase + SmemLayout::kB + stage * kTileBBytes, &tmB, fb, kx, n0, ti.e);
          if (p.prefetch > 0) {
            const int pk = kt + p.prefetch;
            if (pk < p.kt_total) {
              const int pkx = pk * BK - p.k_pad;
              if (pkx >= 0) {
                tma_prefetch_l2_3d(&tmB, pkx, n0, ti.e);
                tma_prefetch_l2_2d(&tmA, pkx, row0);
              }
            } else if (tn < total_tiles && pk - p.kt_total < p.kt_total) {
              const int pkx = (pk - p.kt_total) * BK - p.k_pad;
              if (pkx >= 0) {
                tma_prefetch_l2_3d(&tmB, pkx, tin.nt * BN, tin.e);
                tma_prefetch_l2_2d(&tmA, pkx, row0n);
              }
            }
          }
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
        ti = tin;
        row0 = row0n;
        tn += gridDim.x;
        if (tn < total_tiles) {
          tin = decode_tile(tn, mt_prefix, p.E, p.n_tiles);
          row0n = e_row0[tin.e] + tin.mt * BM;
        }
      }
      if (!ok) {
        // drain: never exit with TMA writes into this CTA's smem in flight
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
          if (issued[s])
            mbar_wait(bar_full + 8 * s, issued_phase[s], &no_abort, &g_err_gemm,
                      kErrDrainTimeout, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool ok = true;
      bool any = false;
      // The issuer needs no tile coordinates: it walks this CTA's quant
      // blocks in order (tiles blockIdx.x, +gridDim.x, ...), one TMEM
      // accumulator buffer per block.  Shared memory filled by TMA is made
      // visible by the full-barrier wait itself; the tcgen05 fence is only
      // needed after the accumulator hand-back, which the epilogue's
      // tcgen05.ld precede.
      const int my_tiles =
          blockIdx.x < total_tiles ? (total_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
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
            umma_i8(d_tmem, ad, bd, kIdesc, (kt > kt0 || k > 0) ? 1u : 0u);
          }
          any = true;
          umma_commit(bar_empty + 8 * stage);
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        umma_commit(bar_accf + 8 * acc);
        if (++acc == NACC) acc = 0, aphase ^= 1;
        if (++qb == p.nq) qb = 0;
      }
      // wait for every issued MMA before TMEM can be released
      if (any) {
        umma_commit(bar_final);
        volatile int no_abort = 0;
        mbar_wait(bar_final, 0, &no_abort, &g_err_gemm, kErrDrainTimeout, 200000000ull);
      }
    }
    __syncwarp();
  } else {
    // ================= epilogue (16 warps) =================
    // TMEM lane quadrant = warp % 4 (hardware rule), column quarter =
    // (warp - 2) / 4: each thread owns one row and 64 columns (one 64-column
    // weight-scale block) of the 128 x 256 tile, so a single Q_A * Q_B factor
    // applies to all of its columns in a quant block.  Four warps share each
    // SM sub-partition, which is what keeps the integer multiply-add pipe
    // busy while the other warps wait for their TMEM loads.
    const int quad = warp & 3;
    const int cq = (warp - 2) >> 2;
    const int rl = quad * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t t_col = (static_cast<uint32_t>(quad * 32) << 16) + cq * 64;
    int acc = 0;
    uint32_t aphase = 0;
    bool ok = true;
    // Every lane of a warp shares one scale row (a 32-row group never
    // straddles a tile_m boundary) and one 64-column weight block, so the
    // factor Q_A * Q_B of a quant block is warp-uniform: lane l holds that
    // of block (qb0 + l), and each block's factor is broadcast by shuffle.
    // The next tile's Q factors and this tile's F factors travel by cp.async
    // into per-thread shared-memory slots while the accumulation runs, so
    // they take no registers from the accumulator.
    // Slots: [Q_A, Q_B] for even local tiles, [Q_A, Q_B] for odd ones, then
    // F_A, F_B; a slot pair is refilled only for the tile after next, so an
    // asynchronous write never meets a pending read of the same slot.
    const uint32_t s_slot = sbase + SmemLayout::kSlots + 4 * (threadIdx.x - 64);
    constexpr uint32_t kSA = SmemLayout::kSlotArray;
    const uint32_t s_fa = s_slot + 4 * kSA;
    const uint32_t s_fb = s_slot + 5 * kSA;
    auto ld_s32 = [](uint32_t a) {
      int v;
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
      return v;
    };
    auto st_s32 = [](uint32_t a, int v) {
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
    };
    // Q_A / Q_B of quant block (qb0 + lane) of tile t, synchronously
    auto tile_q = [&](int t, int qb0) -> int {
      const TileInfo u = decode_tile(t, mt_prefix, p.E, p.n_tiles);
      const int wrow = u.mt * BM + quad * 32;
      const int col = u.nt * BN + cq * 64;
      const int qb = qb0 + lane;
      if (MODE != kHybrid || wrow >= m_rows[u.e] || col >= p.N || qb >= p.nq) return 0;
      const int srow = so_prefix[u.e] + wrow / p.tile_m;
      return __ldg(p.qa + static_cast<int64_t>(srow) * p.q_stride + qb) *
             __ldg(p.qb + (static_cast<int64_t>(u.e) * p.nsb + col / 64) * p.q_stride + qb);
    };
    // Q_A / Q_B of quant blocks 0..31 (one per lane) of tile t, into the
    // slot pair `par` asynchronously
    auto fetch_q = [&](int t, int par) {
      const uint32_t s_qa = s_slot + (2 * par) * kSA, s_qb = s_qa + kSA;
      const int qb0 = 0;
      bool any = false;
      if (MODE == kHybrid && t < total_tiles) {
        const TileInfo u = decode_tile(t, mt_prefix, p.E, p.n_tiles);
        const int wrow = u.mt * BM + quad * 32;
        const int col = u.nt * BN + cq * 64;
        const int qb = qb0 + lane;
        if (wrow < m_rows[u.e] && col < p.N && qb < p.nq) {
          const int srow = so_prefix[u.e] + wrow / p.tile_m;
          cp_async4(s_qa, p.qa + static_cast<int64_t>(srow) * p.q_stride + qb);
          cp_async4(s_qb, p.qb + (static_cast<int64_t>(u.e) * p.nsb + col / 64) * p.q_stride + qb);
          any = true;
        }
      }
      if (!any) {
        st_s32(s_qa, 0);
        st_s32(s_qb, 0);
      }
    };
    auto take_q = [&](int par) {
      cp_async_wait_all();
      const uint32_t s_qa = s_slot + (2 * par) * kSA;
      return ld_s32(s_qa) * ld_s32(s_qa + kSA);
    };
    fetch_q(blockIdx.x, 0);
    int par = 0;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, par ^= 1) {
      int qv = take_q(par);
      fetch_q(t + gridDim.x, par ^ 1);
      {
        // F_A, F_B of this tile (needed only by the output phase)
        const TileInfo ti = decode_tile(t, mt_prefix, p.E, p.n_tiles);
        const int wrow0 = ti.mt * BM + quad * 32;
        const int col0 = ti.nt * BN + cq * 64;
        if (MODE == kHybrid && wrow0 < m_rows[ti.e] && col0 < p.N) {
          const int srow = so_prefix[ti.e] + wrow0 / p.tile_m;
          cp_async4(s_fa, p.fa + static_cast<int64_t>(srow) * p.f_stride);
          cp_async4(s_fb, p.fb + (static_cast<int64_t>(ti.e) * p.nsb + col0 / 64) * p.f_stride);
        }
      }
      int32_t W[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) W[i] = 0;
      // One 16-column chunk in flight per warp: with four epilogue warps on
      // each SM sub-partition the other warps' multiply-adds cover the TMEM
      // load latency, and the single buffer keeps W[64] in registers.  The
      // accumulator buffer goes back to the MMA warp as soon as its last
      // chunk has landed.
      uint32_t P[16];
      for (int qb = 0; qb < p.nq && ok; ++qb) {
        const int q = __shfl_sync(0xffffffffu, qv, qb & 31);
        if ((qb & 31) == 31 && qb + 1 < p.nq) qv = tile_q(t, qb + 1);  // K > 4096
        if (!mbar_wait(bar_accf + 8 * acc, aphase, s_abort, &g_err_gemm, kErrEpilogueTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld16(tmem_base + t_col + acc * BN + 16 * c, P);
          tmem_wait_ld(P);
          if (c == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acce + 8 * acc);
            if (++acc == NACC) acc = 0, aphase ^= 1;
          }
          if (MODE == kHybrid) {
#pragma unroll
            for (int i = 0; i < 16; ++i) W[16 * c + i] += q * static_cast<int32_t>(P[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) W[16 * c + i] += static_cast<int32_t>(P[i]);
          }
        }
      }
      if (!ok) break;
      // ---- convert, scale, round, store ----
      const TileInfo ti = decode_tile(t, mt_prefix, p.E, p.n_tiles);
      const int m_e = m_rows[ti.e];
      const int wrow0 = ti.mt * BM + quad * 32;
      const int lrow = wrow0 + lane;
      const int col0 = ti.nt * BN + cq * 64;
      float f;
      if (MODE == kHybrid) {
        cp_async_wait_all();
        f = __int_as_float(ld_s32(s_fa)) * __int_as_float(ld_s32(s_fb));
      } else if (p.a_row_scale != nullptr) {
        f = lrow < m_e ? __ldg(p.a_row_scale + e_row0[ti.e] + lrow) * __ldg(p.b_expert_scale + ti.e)
                       : 0.f;
      } else {
        f = p.alpha;
      }
      if constexpr (!std::is_same<OutT, int32_t>::value) {
        if (wrow0 + 32 <= m_e && col0 + 64 <= p.N) {
          // All 32 rows belong to this expert: stage the warp's 32 x 64 block
          // in shared memory (64-byte swizzle, conflict-free) and write it
          // with two TMA tensor stores of 32 x 32, so the stores leave as
          // whole lines instead of 32 row fragments per instruction.
          const uint32_t stg = sbase + SmemLayout::kStg + (warp - 2) * SmemLayout::kStgWarpBytes;
          const float* bp =
              HAS_BIAS ? p.bias + static_cast<int64_t>(ti.e) * p.bias_stride + col0 : nullptr;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (lane == 0) bulk_wait_read0();  // the previous store has read the buffer
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t w4[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int c = 32 * h + 8 * j + 2 * i;
                if (HAS_BIAS) {
                  w4[i] = pack2<OutT>(fmaf(static_cast<float>(W[c]), f, __ldg(bp + c)),
                                      fmaf(static_cast<float>(W[c + 1]), f, __ldg(bp + c + 1)));
                } else {
                  w4[i] = pack2<OutT>(__fmul_rn(static_cast<float>(W[c]), f),
                                      __fmul_rn(static_cast<float>(W[c + 1]), f));
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
              tma_store_2d(&tmO, stg, col0 + 32 * h, e_row0[ti.e] + wrow0);
              bulk_commit();
            }
          }
          continue;
        }
      }
      if (!(lrow < m_e && col0 < p.N)) continue;
      const int64_t row_off = static_cast<int64_t>(e_row0[ti.e] + lrow) * p.N + col0;
      const int ncols = min(64, p.N - col0);
      if constexpr (std::is_same<OutT, int32_t>::value) {
        // raw accumulator output (verification mode)
        int32_t* dst = static_cast<int32_t*>(p.out) + row_off;
        (void)f;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          if (4 * c < ncols)
            *reinterpret_cast<int4*>(dst + 4 * c) =
                make_int4(W[4 * c], W[4 * c + 1], W[4 * c + 2], W[4 * c + 3]);
      } else {
        OutT* dst = static_cast<OutT*>(p.out) + row_off;
        const float* bp = HAS_BIAS ? p.bias + static_cast<int64_t>(ti.e) * p.bias_stride + col0
                                   : nullptr;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          if (8 * c >= ncols) continue;
          uint32_t w4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = 8 * c + 2 * i;
            if (HAS_BIAS) {
              w4[i] = pack2<OutT>(fmaf(static_cast<float>(W[j]), f, __ldg(bp + j)),
                                  fmaf(static_cast<float>(W[j + 1]), f, __ldg(bp + j + 1)));
            } else {
              w4[i] = pack2<OutT>(__fmul_rn(static_cast<float>(W[j]), f),
                                  __fmul_rn(static_cast<float>(W[j + 1]), f));
            }
          }
          *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
    cp_async_wait_all();  // no asynchronous copy into shared memory outlives the CTA
    if (lane == 0) bulk_wait0();  // nor a tensor store still reading the staging buffer
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
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

int make_tmap_b(CUtensorMap* m, const int8_t* b, int64_t E, int64_t n, int64_t k) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(n),
                        static_cast<cuuint64_t>(E)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(n * k)};
  cuuint32_t box[3] = {BK, BN, 1};
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

template <int MODE, bool HAS_BIAS, typename OutT>
int launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
             const GemmParams& p, int grid, cudaStream_t st) {
  auto kern = grouped_gemm_kernel<MODE, HAS_BIAS, OutT>;
  const int smem = SmemLayout::bytes(p.E) + 1024;
  static int attr_done[64] = {0};
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || !__atomic_load_n(&attr_done[dev], __ATOMIC_ACQUIRE)) {
    I8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SmemLayout::bytes(kMaxExperts) + 1024));
    if (dev >= 0 && dev < 64) __atomic_store_n(&attr_done[dev], 1, __ATOMIC_RELEASE);
  }
  kern<<<grid, kThreads, smem, st>>>(ta, tb, to, p);
  return check_launch("grouped_gemm_kernel");
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

int launch_gemm(int mode, int out_dtype, bool has_bias, const int8_t* a, const int8_t* b,
                GemmParams p, int64_t E, int64_t sum_m, int64_t n, int64_t k, cudaStream_t st) {
  I8_REQUIRE(out_dtype == I8MOE_BF16 || out_dtype == I8MOE_FP16 || out_dtype == I8MOE_S32,
             "out must be bfloat16 (or float16, or int32 for the raw accumulator)");
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
  CUtensorMap ta, tb;
  rc = make_tmap_a(&ta, a, sum_m, k);
  if (rc) return rc;
  rc = make_tmap_b(&tb, b, E, n, k);
  if (rc) return rc;
  CUtensorMap to = ta;  // the raw int32 output is written without a tensor map
  if (out_dtype != I8MOE_S32) {
    rc = make_tmap_out(&to, p.out, out_dtype, sum_m, n);
    if (rc) return rc;
  }
  p.E = static_cast<int>(E);
  p.sum_m = static_cast<int>(sum_m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.kt_total = static_cast<int>((k + BK - 1) / BK);
  p.k_pad = p.kt_total * BK - p.K;
  p.n_tiles = static_cast<int>((n + BN - 1) / BN);
  const int64_t upper_tiles = ((sum_m + BM - 1) / BM + E) * p.n_tiles;
  {
    const char* pf = getenv("I8MOE_GEMM_PREFETCH");
    p.prefetch = pf ? atoi(pf) : 0;
  }
  const int grid = static_cast<int>(std::min<int64_t>(num_sms(current_device()), upper_tiles));
  if (out_dtype == I8MOE_S32) {
    I8_REQUIRE(!has_bias, "the raw int32 accumulator output takes no bias");
    return mode == kHybrid ? launch_t<kHybrid, false, int32_t>(ta, tb, to, p, grid, st)
                           : launch_t<kPerTensor, false, int32_t>(ta, tb, to, p, grid, st);
  }
  if (mode == kHybrid) {
    if (out_dtype == I8MOE_BF16)
      return has_bias ? launch_t<kHybrid, true, __nv_bfloat16>(ta, tb, to, p, grid, st)
                      : launch_t<kHybrid, false, __nv_bfloat16>(ta, tb, to, p, grid, st);
    return has_bias ? launch_t<kHybrid, true, __half>(ta, tb, to, p, grid, st)
                    : launch_t<kHybrid, false, __half>(ta, tb, to, p, grid, st);
  }
  if (out_dtype == I8MOE_BF16) return launch_t<kPerTensor, false, __nv_bfloat16>(ta, tb, to, p, grid, st);
  return launch_t<kPerTensor, false, __half>(ta, tb, to, p, grid, st);
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

}  // extern "C"
