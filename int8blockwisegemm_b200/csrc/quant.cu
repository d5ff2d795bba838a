// Grouped per-(expert M-tile x 128-K block) INT8 activation quantisation
// with the two-level (Q int32, F fp32) scale factorisation.
//
// Semantics follow int8_hybrid_moe/quant.py of the reference:
//   tile      = rows [eo[e] + i*tm, min(+tm, eo[e+1], M)) x cols [kb*128, +128)
//               of the expert e owning scale row s = so[e] + i      (:169-193)
//   scale     = max(absmax(tile), 1e-10) / 127                      (:200-201)
//   q         = round_half_away(clamp(x / scale, -128, 127))        (:202)
//   F[s, g]   = max(max_{kb in g} |scale[s,kb]|, 1e-12) / q_max     (:84-89)
//   Q[s, kb]  = rint(scale[s, kb] / F[s, g])                        (:90)
// with three row sources: the already permuted activation (:147-209), the
// gathered hidden row hidden[permuted_idx[r] / topk] (:284-357) and
// silu(gate) * up of the w13 output (:440-511).
//
// quant_rows_kernel: one CTA of 256 threads per scale row and run of four
// K-blocks (the row range and gathered source rows are resolved once).
// Every thread loads its 16-byte chunks of the tile straight from global
// memory (rows gathered through permuted_idx for the permute path; gate and
// up halves for the SiLU path) -- a warp instruction covers whole rows, so
// the loads and the int8 stores are coalesced -- and keeps them in
// registers: the tile absmax is reduced by warp shuffles and one CTA barrier,
// and each thread quantises and stores its own chunks.  Four CTAs per SM keep
// ~128 KB of loads in flight.  The block scale of every tile is written into
// the Q buffer; scales_to_qf then factorises each (row, super-group) in place.
//
// x / scale is evaluated as x * (1/scale) (packed f32x2 arithmetic); a
// product farther than 3e-5 from a rounding tie rounds exactly as the IEEE
// quotient does (the product is within 1.6e-5 of x/scale, the IEEE quotient
// within 3.9e-6, for |x/scale| <= 128); the rare elements closer to a tie (or
// not finite) are recomputed with the IEEE division.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "quant_math.cuh"

namespace i8moe {

static __device__ unsigned g_err_quant;

int read_quant_error(uint32_t* w, int clear) {
  unsigned v = 0;
  I8_CUDA(cudaMemcpyFromSymbol(&v, g_err_quant, sizeof(v)));
  if (clear) {
    unsigned z = 0;
    I8_CUDA(cudaMemcpyToSymbol(g_err_quant, &z, sizeof(z)));
  }
  *w = v;
  return I8MOE_OK;
}

namespace {

constexpr int kMaxE = 2048;
constexpr int kQuantThreads = 256;

enum Mode { kDirect = 0, kGather = 1, kSilu = 2 };

struct QuantArgs {
  const void* src;     // direct [M, K], gather [n_src, K], silu [M, 2K]
  int64_t src_stride;  // elements per source row
  int64_t src_rows;    // rows of the source
  int M;               // rows of qA
  int K;               // quantised columns
  int topk;            // gather mode
  const int32_t* pidx;
  const int32_t* eo;  // [E+1]
  const int32_t* so;  // [E+1]
  int E;
  int Kb;
  int8_t* qA;
  float* scale_out;  // [rows, Kb] block scales (the Q buffer, rewritten later)
};

// Largest e in [0, E) with so[e] <= s (so non-decreasing, so[E] > s): the
// expert owning scale row s.  32-ary search by one warp.
__device__ __forceinline__ int expert_of_scale_row(const int32_t* so, int E, int s, int lane) {
  int lo = 0, hi = E;
  while (hi - lo > 1) {
    const int step = (hi - lo + 31) / 32;
    const int idx = lo + lane * step;  // candidates lo, lo+step, ... below hi
    const unsigned m = __ballot_sync(0xffffffffu, idx < hi && __ldg(so + idx) <= s);
    const int last = 31 - __clz(m);  // lane 0 reads so[lo] <= s, so m != 0
    lo += last * step;
    hi = min(lo + step, hi);
  }
  return lo;
}

template <typename T, int TM, int MODE>
struct RowsTile {
  static constexpr int EPC = 16 / sizeof(T);       // elements per 16-byte chunk
  static constexpr int CPR = 128 / EPC;            // chunks per 128-column row segment
  static constexpr int RPW = 32 / CPR;             // rows per warp instruction
  static constexpr int RPP = RPW * (kQuantThreads / 32);  // rows per pass of the CTA
  static constexpr int NP = TM / RPP;              // passes = chunks per thread
  static constexpr int MIN_BLOCKS = (NP * (MODE == kSilu ? 2 : 1) > 8) ? 2 : 4;
  static_assert(TM % RPP == 0, "tile rows");
};

constexpr int kKbPerCta = 4;  // K-blocks of one scale row handled by one CTA

// OFF32: every source and qA element offset fits in 31 bits (checked by the
// launcher), so addresses are formed with 32-bit multiply-adds -- fewer
// instructions per chunk than 64-bit products (default shape: 104.8 ->
// 98.8 us).
template <typename T, int TM, int MODE, bool OFF32>
__global__ void __launch_bounds__(kQuantThreads, (RowsTile<T, TM, MODE>::MIN_BLOCKS))
    quant_rows_kernel(QuantArgs a) {
  using TL = RowsTile<T, TM, MODE>;
  constexpr int EPC = TL::EPC, CPR = TL::CPR, RPW = TL::RPW, RPP = TL::RPP, NP = TL::NP;
  __shared__ float s_red[2][kQuantThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int groups = (a.Kb + kKbPerCta - 1) / kKbPerCta;
  const int s = blockIdx.x / groups;
  const int kb0 = (blockIdx.x - s * groups) * kKbPerCta;
  if (s >= __ldg(a.so + a.E)) return;  // past the last scale row of this routing
  // the tile rows (and, for the gather, their source rows) are shared by all
  // K-blocks of the scale row: resolved once per CTA
  const int e = expert_of_scale_row(a.so, a.E, s, lane);
  const int so_e = __ldg(a.so + e);
  const int row_start = __ldg(a.eo + e) + (s - so_e) * TM;
  const int row_end = min(min(__ldg(a.eo + e + 1), a.M), row_start + TM);
  const int rows = row_end - row_start;
  if (!(so_e <= s && s < __ldg(a.so + e + 1) && row_start >= 0)) {
    if (threadIdx.x == 0) atomicOr(&g_err_quant, kErrBadIndex);  // inconsistent offsets
    return;
  }
  const int cc = lane % CPR;
  const T* src = static_cast<const T*>(a.src);
  // source row of this thread's row in each pass, -1 if none (32-bit: the
  // eight rows stay in registers across the K-blocks without spilling)
  int32_t src_row[NP];
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int r = j * RPP + warp * RPW + lane / CPR;
    src_row[j] = -1;
    if (r < rows) {
      int srow = row_start + r;
      if (MODE == kGather) srow = __ldg(a.pidx + srow) / a.topk;
      src_row[j] = srow;
    }
  }
  const int kb1 = min(kb0 + kKbPerCta, a.Kb);
  for (int kb = kb0; kb < kb1; ++kb) {
    const int col = kb * 128 + cc * EPC;
    const bool col_ok = col < a.K;
    // ---- load this thread's chunks (all passes in flight together) ----
    uint4 v[NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      v[j] = make_uint4(0u, 0u, 0u, 0u);
      if (src_row[j] >= 0 && col_ok) {
        const T* p = OFF32 ? src + (static_cast<uint32_t>(src_row[j]) *
                                        static_cast<uint32_t>(a.src_stride) +
                                    static_cast<uint32_t>(col))
                           : src + static_cast<int64_t>(src_row[j]) * a.src_stride + col;
        if (MODE == kSilu) {
          const uint4 g = __ldg(reinterpret_cast<const uint4*>(p));
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(p + a.K));
          v[j] = silu_mul_chunk<T>(g, u);
        } else {
          v[j] = __ldg(reinterpret_cast<const uint4*>(p));
        }
      }
    }
    // ---- tile absmax (NaN-ignoring, as tl.max / fmaxf) ----
    float m = 0.0f;
    if constexpr (sizeof(T) == 2) {
      uint32_t acc = 0u;
#pragma unroll
      for (int j = 0; j < NP; ++j) acc = absmax16_acc<T>(acc, v[j]);
      m = absmax16_value<T>(acc);
    } else {
#pragma unroll
      for (int j = 0; j < NP; ++j) m = fmaxf(m, chunk_absmax<T>(v[j]));
    }
    const unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
    const int buf = (kb - kb0) & 1;  // alternate, so one barrier per K-block suffices
    if (lane == 0) s_red[buf][warp] = __uint_as_float(mb);
    __syncthreads();
    float amax = s_red[buf][0];
#pragma unroll
    for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, s_red[buf][w]);
    const float scale = __fdiv_rn(fmaxf(amax, 1e-10f), 127.0f);
    if (tid == 0) a.scale_out[static_cast<int64_t>(s) * a.Kb + kb] = scale;
    // ---- quantise and store ----
    if (!col_ok) continue;
    if constexpr (sizeof(T) == 2) {
      const QuantInv qi = quant_inv(scale);
      // Every chunk is stored from the bracketed fast path; the rare chunks
      // near a rounding tie (or not finite) are recomputed exactly and stored
      // again after one branch per K-block, so the common path has no
      // per-chunk branch.  row_start + r < row_end <= M for every r < rows:
      // the row range was validated above.
      int8_t* dst = OFF32 ? a.qA + (static_cast<uint32_t>(row_start) * static_cast<uint32_t>(a.K) +
                                    static_cast<uint32_t>(col))
                          : a.qA + static_cast<int64_t>(row_start) * a.K + col;
      auto row_off = [&](int r) -> int64_t {
        return OFF32 ? static_cast<int64_t>(static_cast<uint32_t>(r) * static_cast<uint32_t>(a.K))
                     : static_cast<int64_t>(r) * a.K;
      };
      unsigned redo = 0u;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int r = j * RPP + warp * RPW + lane / CPR;
        uint2 q;
        const bool fast = quant_chunk_bracket<T>(v[j], qi, q);
        if (r < rows) {
          *reinterpret_cast<uint2*>(dst + row_off(r)) = q;
          if (!fast) redo |= 1u << j;
        }
      }
      if (redo) {
#pragma unroll
        for (int j = 0; j < NP; ++j) {
          const int r = j * RPP + warp * RPW + lane / CPR;
          if (redo & (1u << j))
            *reinterpret_cast<uint2*>(dst + row_off(r)) =
                quant_chunk_exact16<T>(v[j], scale);
        }
      }
    } else {
      const float inv = __frcp_rn(scale);
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int r = j * RPP + warp * RPW + lane / CPR;
        if (r >= rows) continue;
        uint32_t words[EPC / 4];
        if (!quant_chunk_fast<T>(v[j], inv, words)) quant_chunk_exact<T>(v[j], inv, scale, words);
        if (static_cast<unsigned>(row_start + r) >= static_cast<unsigned>(a.M)) {
          atomicOr(&g_err_quant, kErrBadIndex);  // never store outside qA
          continue;
        }
        *reinterpret_cast<uint32_t*>(a.qA + static_cast<int64_t>(row_start + r) * a.K + col) =
            words[0];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Weight preparation (reference bench_int8_hybrid_moe.py:98-120): blockwise
// INT8 weights, one CTA per (expert, 64-row, 128-column) block.  Rows and
// columns past the tensor are the reference's zero padding: they join the
// absmax as zeros and are not stored.
// ---------------------------------------------------------------------------
constexpr int kWBlockN = 64, kWBlockK = 128;

template <typename T>
__global__ void __launch_bounds__(kQuantThreads) weight_quant_kernel(const T* __restrict__ w,
                                                                     int N, int K, int nb, int kb,
                                                                     int8_t* __restrict__ q,
                                                                     float* __restrict__ scale) {
  constexpr int EPC = 16 / sizeof(T);
  constexpr int CPR = kWBlockK / EPC;              // chunks per row of the block
  constexpr int RPP = kQuantThreads / CPR;         // rows per pass
  constexpr int NP = kWBlockN / RPP;               // chunks per thread
  __shared__ float s_red[kQuantThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int blk = blockIdx.x;
  const int bk = blk % kb, bn = (blk / kb) % nb, e = blk / (kb * nb);
  const int col = bk * kWBlockK + (tid % CPR) * EPC;
  const int64_t base = static_cast<int64_t>(e) * N * K;
  uint4 v[NP];
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int row = bn * kWBlockN + j * RPP + tid / CPR;
    v[j] = make_uint4(0u, 0u, 0u, 0u);
    if (row < N && col < K)
      v[j] = __ldg(reinterpret_cast<const uint4*>(w + base + static_cast<int64_t>(row) * K + col));
  }
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < NP; ++j) m = fmaxf(m, chunk_absmax<T>(v[j]));
  const unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
  if (lane == 0) s_red[warp] = __uint_as_float(mb);
  __syncthreads();
  float amax = s_red[0];
#pragma unroll
  for (int i = 1; i < kQuantThreads / 32; ++i) amax = fmaxf(amax, s_red[i]);
  const float sc = __fdiv_rn(fmaxf(amax, 1e-10f), 127.0f);
  const float inv = __frcp_rn(sc);
  if (tid == 0) scale[blk] = sc;
  if (col >= K) return;
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int row = bn * kWBlockN + j * RPP + tid / CPR;
    if (row >= N) continue;
    uint32_t words[EPC / 4];
    // the fast rounding equals rint wherever it does not defer (no ties)
    if (!quant_chunk_fast<T>(v[j], inv, words)) quant_chunk_exact_rne<T>(v[j], sc, words);
    int8_t* dst = q + base + static_cast<int64_t>(row) * K + col;
    if constexpr (EPC == 8) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(words[0], words[1]);
    } else {
      *reinterpret_cast<uint32_t*>(dst) = words[0];
    }
  }
}

// Q/F factorisation of fp32 block scales, one warp per (row, super-group).
// `scale` and `Q` may alias (in-place): every lane rewrites only the entries
// it read, after the group maximum has been reduced.  When `rows_dev` is
// non-null the row count is read from it (rows beyond it are skipped).
__global__ void scales_to_qf(const float* scale, int rows, const int32_t* rows_dev, int kb,
                             float qmax, int sg, int nsg, int32_t* Q, float* F) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nrows = rows_dev ? min(rows, *rows_dev) : rows;
  if (warp >= nrows * nsg) return;
  const int r = warp / nsg, g = warp % nsg;
  const int lo = g * sg, hi = min(lo + sg, kb);
  float m = 0.0f;
  for (int k = lo + lane; k < hi; k += 32) m = fmaxf(m, fabsf(scale[static_cast<int64_t>(r) * kb + k]));
  m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
  const float fg = __fdiv_rn(fmaxf(m, 1e-12f), qmax);
  for (int k = lo + lane; k < hi; k += 32) {
    const float v = scale[static_cast<int64_t>(r) * kb + k];
    Q[static_cast<int64_t>(r) * kb + k] = __float2int_rz(rintf(__fdiv_rn(v, fg)));
  }
  if (lane == 0) F[static_cast<int64_t>(r) * nsg + g] = fg;
}

// so[0] = 0, so[e+1] = so[e] + ceil((eo[e+1]-eo[e]) / tm); one CTA.
__global__ void __launch_bounds__(1024) scale_offsets_kernel(const int32_t* eo, int E, int tm,
                                                             int32_t* so) {
  __shared__ int s_warp[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (E + 1023) / 1024;
  const int lo = tid * per;
  int loc = 0;
  for (int i = 0; i < per; ++i)
    if (lo + i < E) loc += (eo[lo + i + 1] - eo[lo + i] + tm - 1) / tm;
  int x = loc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;
  }
  __syncthreads();
  int pre = x - loc + (warp > 0 ? s_warp[warp - 1] : 0);
  for (int i = 0; i < per; ++i) {
    if (lo + i < E) {
      so[lo + i] = pre;
      pre += (eo[lo + i + 1] - eo[lo + i] + tm - 1) / tm;
    }
  }
  if (E == 0) {
    if (tid == 0) so[0] = 0;
  } else if (lo < E && lo + per >= E) {
    so[E] = pre;
  }
}

template <typename T, int TM, int MODE>
int launch_quant_t(const QuantArgs& a, int rows_upper, cudaStream_t st) {
  const int64_t items = static_cast<int64_t>(rows_upper) * ((a.Kb + kKbPerCta - 1) / kKbPerCta);
  if (items == 0) return I8MOE_OK;
  I8_REQUIRE(items < (int64_t(1) << 31), "quant: too many tiles");
  // every element offset (source rows x stride + 128-column padding, and
  // qA rows x K) below 2^31: 32-bit address arithmetic
  constexpr int64_t kLim = int64_t(1) << 31;
  const bool off32 = a.src_rows * a.src_stride + 128 < kLim &&
                     static_cast<int64_t>(a.M) * a.K + 128 < kLim;
  if (off32)
    quant_rows_kernel<T, TM, MODE, true><<<static_cast<unsigned>(items), kQuantThreads, 0, st>>>(a);
  else
    quant_rows_kernel<T, TM, MODE, false><<<static_cast<unsigned>(items), kQuantThreads, 0, st>>>(a);
  return check_launch("quant");
}

template <int MODE>
int launch_quant_mode(int dtype, int tm, const QuantArgs& a, int rows_upper, cudaStream_t st) {
  if (dtype == I8MOE_BF16) {
    return tm == 64 ? launch_quant_t<__nv_bfloat16, 64, MODE>(a, rows_upper, st)
                    : launch_quant_t<__nv_bfloat16, 128, MODE>(a, rows_upper, st);
  } else if (dtype == I8MOE_FP16) {
    return tm == 64 ? launch_quant_t<__half, 64, MODE>(a, rows_upper, st)
                    : launch_quant_t<__half, 128, MODE>(a, rows_upper, st);
  }
  if constexpr (MODE == kSilu) {
    return set_error(I8MOE_ERR_INVALID, "quant: the SiLU path takes bfloat16 or float16");
  } else {
    return tm == 64 ? launch_quant_t<float, 64, MODE>(a, rows_upper, st)
                    : launch_quant_t<float, 128, MODE>(a, rows_upper, st);
  }
}

// src: direct [M, K], gather [n_src, K] (rows picked by pidx / topk), silu
// [M, 2K] (gate columns then up columns).
int launch_quant(int mode, const void* src, int dtype, int64_t src_rows, int64_t src_cols,
                 int64_t M, int64_t K, const int32_t* pidx, int64_t topk, const int32_t* eo,
                 int64_t E, int64_t tm, int64_t block_k, int64_t q_max, int64_t sg, int8_t* qA,
                 int32_t* Q, float* F, int32_t* so, int so_ready, cudaStream_t st) {
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16 || dtype == I8MOE_FP32,
             "quant: A must be float32, float16 or bfloat16");
  I8_REQUIRE(block_k == 128, "quant: block_k must be 128 (the only quant block the GEMM reads)");
  I8_REQUIRE(tm == 64 || tm == 128, "quant: tile_m must be 64 or 128");
  I8_REQUIRE(sg > 0 && q_max > 0, "quant: super_group_size and q_max must be positive");
  I8_REQUIRE(E >= 1 && E <= kMaxE, "quant: number of experts must be in [1, %d]", kMaxE);
  I8_REQUIRE(K % 8 == 0, "quant: K must be a multiple of 8");
  I8_REQUIRE(M >= 0 && M < (int64_t(1) << 31), "quant: bad M");
  const int64_t Kb = (K + block_k - 1) / block_k;
  I8_REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0, "quant: source must be 16-byte aligned");
  I8_REQUIRE(reinterpret_cast<uintptr_t>(qA) % 8 == 0, "quant: qA must be 8-byte aligned");
  if (!so_ready) {
    scale_offsets_kernel<<<1, 1024, 0, st>>>(eo, static_cast<int>(E), static_cast<int>(tm), so);
    int rc = check_launch("scale_offsets");
    if (rc) return rc;
  }
  const int64_t rows_upper = (M + tm - 1) / tm + E;
  if (M == 0 || K == 0 || src_rows == 0) return I8MOE_OK;
  QuantArgs a{};
  a.src = src;
  a.src_stride = src_cols;
  a.src_rows = src_rows;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.topk = static_cast<int>(topk);
  a.pidx = pidx;
  a.eo = eo;
  a.so = so;
  a.E = static_cast<int>(E);
  a.Kb = static_cast<int>(Kb);
  a.qA = qA;
  a.scale_out = reinterpret_cast<float*>(Q);  // rewritten in place by scales_to_qf
  const int ru = static_cast<int>(std::min<int64_t>(rows_upper, INT32_MAX / std::max<int64_t>(Kb, 1)));
  const int t = static_cast<int>(tm);
  int rc;
  if (mode == kDirect) rc = launch_quant_mode<kDirect>(dtype, t, a, ru, st);
  else if (mode == kGather) rc = launch_quant_mode<kGather>(dtype, t, a, ru, st);
  else rc = launch_quant_mode<kSilu>(dtype, t, a, ru, st);
  if (rc) return rc;
  const int nsg = static_cast<int>((Kb + sg - 1) / sg);
  const int64_t warps = static_cast<int64_t>(ru) * nsg;
  scales_to_qf<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const float*>(Q), ru, so + E, static_cast<int>(Kb), static_cast<float>(q_max),
      static_cast<int>(sg), nsg, Q, F);
  return check_launch("quant");
}

}  // namespace

// Q/F factorisation of `rows_upper` rows of raw block scales (rows past
// *rows_dev, when given, are skipped), in place over Q.
int launch_scales_to_qf(const float* scale, int64_t rows_upper, const int32_t* rows_dev,
                        int64_t kb, int64_t q_max, int64_t sg, int32_t* Q, float* F,
                        cudaStream_t st) {
  I8_REQUIRE(rows_upper >= 0 && kb >= 0 && sg > 0 && q_max > 0, "quantize_scales: bad arguments");
  if (rows_upper == 0 || kb == 0) return I8MOE_OK;
  const int64_t nsg = (kb + sg - 1) / sg;
  const int64_t warps = rows_upper * nsg;
  scales_to_qf<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(
      scale, static_cast<int>(rows_upper), rows_dev, static_cast<int>(kb),
      static_cast<float>(q_max), static_cast<int>(sg), static_cast<int>(nsg), Q, F);
  return check_launch("scales_to_qf");
}

}  // namespace i8moe

using namespace i8moe;

extern "C" {

int i8moe_scale_offsets(const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                        int32_t* scale_offsets, i8moe_stream_t stream) {
  I8_REQUIRE(n_expert >= 0 && tile_m > 0, "scale_offsets: bad arguments");
  scale_offsets_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      expert_offsets, static_cast<int>(n_expert), static_cast<int>(tile_m), scale_offsets);
  return check_launch("scale_offsets");
}

int i8moe_quant_grouped(const void* A, int dtype, int64_t M, int64_t K,
                        const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                        int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                        int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                        i8moe_stream_t stream) {
  return launch_quant(kDirect, A, dtype, M, K, M, K, nullptr, 1, expert_offsets, n_expert, tile_m,
                      block_k, q_max, super_group_size, qA, Q, F, scale_offsets,
                      scale_offsets_ready, static_cast<cudaStream_t>(stream));
}

int i8moe_quant_permute(const void* hidden, int dtype, int64_t n_token, int64_t K,
                        const int32_t* permuted_idx, int64_t M, int64_t topk,
                        const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                        int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                        int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                        i8moe_stream_t stream) {
  I8_REQUIRE(topk > 0, "quant_permute: topk must be positive");
  return launch_quant(kGather, hidden, dtype, n_token, K, M, K, permuted_idx, topk, expert_offsets,
                      n_expert, tile_m, block_k, q_max, super_group_size, qA, Q, F,
                      scale_offsets, scale_offsets_ready, static_cast<cudaStream_t>(stream));
}

int i8moe_quant_silu(const void* mm1, int dtype, int64_t M, int64_t N,
                     const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                     int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                     int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                     i8moe_stream_t stream) {
  return launch_quant(kSilu, mm1, dtype, M, 2 * N, M, N, nullptr, 1, expert_offsets, n_expert,
                      tile_m, block_k, q_max, super_group_size, qA, Q, F, scale_offsets,
                      scale_offsets_ready, static_cast<cudaStream_t>(stream));
}

int i8moe_quantize_weights(const void* w, int dtype, int64_t n_expert, int64_t n, int64_t k,
                           int64_t block_n, int64_t block_k, int8_t* q, float* scale,
                           i8moe_stream_t stream) {
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16 || dtype == I8MOE_FP32,
             "quantize_weights: w must be float32, float16 or bfloat16");
  I8_REQUIRE(block_n == kWBlockN && block_k == kWBlockK,
             "quantize_weights: blocks of 64 x 128 (the GEMM's weight-scale blocks) only");
  I8_REQUIRE(n_expert >= 0 && n > 0 && k > 0, "quantize_weights: bad shape");
  I8_REQUIRE(k % (dtype == I8MOE_FP32 ? 4 : 8) == 0, "quantize_weights: K must allow 16-byte rows");
  I8_REQUIRE((reinterpret_cast<uintptr_t>(w) % 16 == 0) && (reinterpret_cast<uintptr_t>(q) % 8 == 0),
             "quantize_weights: w must be 16-byte and q 8-byte aligned");
  const int64_t nb = (n + kWBlockN - 1) / kWBlockN, kb = (k + kWBlockK - 1) / kWBlockK;
  const int64_t blocks = n_expert * nb * kb;
  I8_REQUIRE(blocks < (int64_t(1) << 31) && n_expert * n * k < (int64_t(1) << 62),
             "quantize_weights: tensor too large");
  if (blocks == 0) return I8MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
  const int N = static_cast<int>(n), K = static_cast<int>(k);
  if (dtype == I8MOE_BF16)
    weight_quant_kernel<__nv_bfloat16><<<g, kQuantThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(w), N, K, static_cast<int>(nb), static_cast<int>(kb), q, scale);
  else if (dtype == I8MOE_FP16)
    weight_quant_kernel<__half><<<g, kQuantThreads, 0, st>>>(
        static_cast<const __half*>(w), N, K, static_cast<int>(nb), static_cast<int>(kb), q, scale);
  else
    weight_quant_kernel<float><<<g, kQuantThreads, 0, st>>>(
        static_cast<const float*>(w), N, K, static_cast<int>(nb), static_cast<int>(kb), q, scale);
  return check_launch("quantize_weights");
}

int i8moe_quantize_scales(const float* scale, int64_t rows, int64_t kb, int64_t q_max,
                          int64_t super_group_size, int32_t* Q, float* F,
                          i8moe_stream_t stream) {
  I8_REQUIRE(rows >= 0 && kb >= 0 && super_group_size > 0 && q_max > 0,
             "quantize_scales: bad arguments");
  if (rows == 0 || kb == 0) return I8MOE_OK;
  const int64_t nsg = (kb + super_group_size - 1) / super_group_size;
  const int64_t warps = rows * nsg;
  const int grid = static_cast<int>((warps * 32 + 255) / 256);
  scales_to_qf<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      scale, static_cast<int>(rows), nullptr, static_cast<int>(kb), static_cast<float>(q_max),
      static_cast<int>(super_group_size), static_cast<int>(nsg), Q, F);
  return check_launch("quantize_scales");
}

}  // extern "C"
