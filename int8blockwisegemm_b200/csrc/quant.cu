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
// quant_kernel: a persistent grid (one CTA per SM) walks the (scale row,
// K-block) tiles round-robin.  Warp 16 is the producer: it brings every tile
// into a NS-deep shared-memory ring by TMA -- a dense 2-D box for contiguous
// sources, four-row tile::gather4 boxes (row indices from permuted_idx) for
// the permute gather -- and publishes the tile's row range next to it.  Warps
// 0..15 form four independent consumer groups of four warps; group g takes
// every fourth tile: pass 1 reduces the tile absmax from shared memory (warp
// shuffles + a group named barrier), pass 2 quantises and stores the int8
// rows, then the stage is released to the producer.  No CTA-wide barrier
// sits on the hot path.  The block scale of every tile is written into the Q
// buffer; scales_to_qf then factorises each (row, super-group) in place.
//
// x / scale is evaluated as x * (1/scale) (packed f32x2 arithmetic); a
// product farther than 3e-5 from a rounding tie rounds exactly as the IEEE
// quotient does (the product is within 1.6e-5 of x/scale, the IEEE quotient
// within 3.9e-6, for |x/scale| <= 128); the rare elements closer to a tie (or
// not finite) are recomputed with the IEEE division.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
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

constexpr int kGroupThreads = 128;
constexpr int kMaxE = 2048;

enum Mode { kDirect = 0, kGather = 1, kSilu = 2 };

struct QuantArgs {
  int M;           // rows of qA
  int K;           // quantised columns
  int topk;        // gather mode
  const int32_t* pidx;
  const int32_t* eo;  // [E+1]
  const int32_t* so;  // [E+1]
  int E;
  int Kb;
  int8_t* qA;
  float* scale_out;  // [rows, Kb] block scales (the Q buffer, rewritten later)
};

struct TileInfo {
  int s, kb, row_start, rows;
};

// Bounded spin until the producer has issued item `it`.
__device__ __forceinline__ bool wait_issued(const int* s_issued, int it, volatile int* abort) {
  const volatile int* p = s_issued;
  if (*p > it) return true;
  const uint64_t t0 = globaltimer();
  while (*p <= it) {
    if (*abort) return false;
    if (globaltimer() - t0 > I8MOE_WAIT_TIMEOUT_NS) {
      *abort = 1;
      atomicOr(&g_err_quant, kErrEpilogueTimeout);
      return false;
    }
    __nanosleep(200);
  }
  __threadfence_block();
  return true;
}

__device__ __forceinline__ int find_expert(const int* s_so, int E, int s) {
  int lo = 0, hi = E;  // last e in [0, E) with so[e] <= s
  while (lo + 1 < hi) {
    const int mid = (lo + hi) >> 1;
    if (s_so[mid] <= s) lo = mid; else hi = mid;
  }
  return lo;
}


template <typename T, int TM, int MODE>
struct QuantTile {
  static constexpr int EPC = 16 / sizeof(T);      // elements per 16-B chunk
  static constexpr int CPR = 128 / EPC;           // chunks per 128-wide row segment
  static constexpr int ROWB = 128 * sizeof(T);    // bytes of one row segment
  static constexpr int TILEB = TM * ROWB;
  static constexpr int STAGEB = TILEB * (MODE == kSilu ? 2 : 1);
  // ~96 KB of stages (two CTAs per SM) for the 16/32 KB tiles, the 64 KB
  // SiLU tiles take 192 KB (one CTA per SM).
  static constexpr int NS = STAGEB <= 16 * 1024 ? 6 : (STAGEB <= 64 * 1024 ? 3 : 1);
  static constexpr int GROUPS = NS < 4 ? NS : 4;            // consumer groups of 4 warps
  static constexpr int THREADS = GROUPS * kGroupThreads + 32;  // + producer warp
  static constexpr int CHUNKS = TM * CPR;
  static constexpr int CPT = CHUNKS / kGroupThreads;  // chunks per consumer thread
  static_assert(CHUNKS % kGroupThreads == 0, "tile chunks");
};

template <typename T, int TM, int MODE>
__global__ void __launch_bounds__(QuantTile<T, TM, MODE>::THREADS, 1)
    quant_kernel(const __grid_constant__ CUtensorMap tmap, QuantArgs a) {
  using TL = QuantTile<T, TM, MODE>;
  constexpr int EPC = TL::EPC, CPR = TL::CPR, NS = TL::NS, CPT = TL::CPT;
  constexpr int kGroups = TL::GROUPS, kThreads = TL::THREADS;
  constexpr int kConsumerThreads = kGroups * kGroupThreads;

  extern __shared__ __align__(1024) uint8_t qsm_raw[];
  uint8_t* stage_mem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(qsm_raw) + 1023) & ~uintptr_t(1023));
  int* s_so = reinterpret_cast<int*>(stage_mem + NS * TL::STAGEB);
  int* s_eo = s_so + (a.E + 1);
  __shared__ __align__(8) uint64_t s_full[NS];
  __shared__ __align__(8) uint64_t s_empty[NS];
  __shared__ TileInfo s_info[NS];
  __shared__ float s_red[4][2][4];
  __shared__ int s_abort;
  // Items handed to TMA so far.  Consumer groups take stages out of order, so
  // a group may only wait on a stage's barrier once its own item has been
  // issued there: then the barrier is pending exactly that item's phase and
  // the parity wait cannot be satisfied by an older phase.
  __shared__ int s_issued;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i <= a.E; i += kThreads) {
    s_so[i] = __ldg(a.so + i);
    s_eo[i] = __ldg(a.eo + i);
  }
  if (tid == 0) {
    s_abort = 0;
    s_issued = 0;
    for (int st = 0; st < NS; ++st) {
      mbar_init(smem_u32(&s_full[st]), 1);
      mbar_init(smem_u32(&s_empty[st]), kGroupThreads / 32);
    }
    mbar_fence_init();
  }
  __syncthreads();
  const int total_items = s_so[a.E] * a.Kb;
  const int n_items = blockIdx.x < total_items
                          ? (total_items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  if (warp == kConsumerThreads / 32) {
    // ======================= producer warp =======================
    if (lane == 0) tma_prefetch_desc(&tmap);
    int last = -1;
    bool ok = true;
    // gather rows of the next item are loaded one item ahead
    int src[4] = {0, 0, 0, 0};
    auto item_rows = [&](int it, int& s, int& kb, int& row_start, int& row_end) {
      const int g = blockIdx.x + it * gridDim.x;
      s = g / a.Kb;
      kb = g - s * a.Kb;
      const int e = find_expert(s_so, a.E, s);
      row_start = s_eo[e] + (s - s_so[e]) * TM;
      row_end = min(min(s_eo[e + 1], a.M), row_start + TM);
    };
    auto load_src = [&](int it) {
      int s, kb, rs, re;
      item_rows(it, s, kb, rs, re);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = rs + 4 * lane + q;
        src[q] = (4 * lane < TM && r < re) ? __ldg(a.pidx + r) / a.topk : 0;
      }
    };
    if (MODE == kGather && n_items > 0) load_src(0);
    for (int it = 0; it < n_items && ok; ++it) {
      const int st = it % NS;
      const uint32_t par = static_cast<uint32_t>(((it / NS) & 1) ^ 1);
      if (!mbar_wait(smem_u32(&s_empty[st]), par, &s_abort, &g_err_quant, kErrProducerTimeout)) {
        ok = false;
        break;
      }
      int s, kb, row_start, row_end;
      item_rows(it, s, kb, row_start, row_end);
      const int col = kb * 128;
      const uint32_t bar = smem_u32(&s_full[st]);
      const uint32_t dst = smem_u32(stage_mem + st * TL::STAGEB);
      if (lane == 0) s_info[st] = TileInfo{s, kb, row_start, row_end - row_start};
      __syncwarp();
      if (MODE == kGather) {
        if (lane == 0) mbar_arrive_expect_tx(bar, TL::STAGEB);
        __syncwarp();
        if (4 * lane < TM)
          tma_gather4(dst + lane * 4 * TL::ROWB, &tmap, bar, col, src[0], src[1], src[2], src[3]);
        if (it + 1 < n_items) load_src(it + 1);
      } else if (lane == 0) {
        mbar_arrive_expect_tx(bar, TL::STAGEB);
        tma_load_2d(dst, &tmap, bar, col, row_start);
        if (MODE == kSilu) tma_load_2d(dst + TL::TILEB, &tmap, bar, col + a.K, row_start);
      }
      last = it;
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        *reinterpret_cast<volatile int*>(&s_issued) = it + 1;
      }
    }
    if (!ok && lane == 0) {
      // never exit with TMA writes into this CTA's shared memory in flight
      int no_abort = 0;
      for (int it = max(0, last - NS + 1); it <= last; ++it)
        mbar_wait(smem_u32(&s_full[it % NS]), static_cast<uint32_t>((it / NS) & 1), &no_abort,
                  &g_err_quant, kErrDrainTimeout, 200000000ull);
    }
    return;
  }

  // ======================= consumer groups =======================
  const int grp = warp >> 2;
  const int gtid = tid & (kGroupThreads - 1);
  const int gwarp = warp & 3;
  int parity_red = 0;
  for (int it = grp; it < n_items; it += kGroups) {
    const int st = it % NS;
    if (!wait_issued(&s_issued, it, &s_abort)) break;
    if (!mbar_wait(smem_u32(&s_full[st]), static_cast<uint32_t>((it / NS) & 1), &s_abort,
                   &g_err_quant, kErrEpilogueTimeout))
      break;
    const TileInfo ti = s_info[st];
    uint8_t* tile = stage_mem + st * TL::STAGEB;
    const int col0 = ti.kb * 128;

    // ---- pass 1: (SiLU: act = dtype(silu(g)) * up, written back over g)
    //      and the tile absmax (NaN-ignoring, as tl.max / fmaxf) ----
    float m = 0.0f;
#pragma unroll 1
    for (int j = 0; j < CPT; ++j) {
      const int c = gtid + j * kGroupThreads;
      const int r = c / CPR, cc = c % CPR;
      if (r < ti.rows && col0 + cc * EPC < a.K) {
        uint4* gp = reinterpret_cast<uint4*>(tile + r * TL::ROWB + cc * 16);
        uint4 v = *gp;
        if (MODE == kSilu) {
          const uint4 u = *reinterpret_cast<const uint4*>(tile + TL::TILEB + r * TL::ROWB + cc * 16);
          v = silu_mul_chunk<T>(v, u);
          *gp = v;
        }
        m = fmaxf(m, chunk_absmax<T>(v));
      }
    }
    const unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
    if (lane == 0) s_red[grp][parity_red][gwarp] = __uint_as_float(mb);
    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(kGroupThreads) : "memory");
    float amax = s_red[grp][parity_red][0];
#pragma unroll
    for (int w = 1; w < 4; ++w) amax = fmaxf(amax, s_red[grp][parity_red][w]);
    parity_red ^= 1;
    const float scale = __fdiv_rn(fmaxf(amax, 1e-10f), 127.0f);
    const float inv = __frcp_rn(scale);
    if (gtid == 0) a.scale_out[static_cast<int64_t>(ti.s) * a.Kb + ti.kb] = scale;

    // ---- pass 2: quantise and store ----
#pragma unroll 1
    for (int j = 0; j < CPT; ++j) {
      const int c = gtid + j * kGroupThreads;
      const int r = c / CPR, cc = c % CPR;
      const int col = col0 + cc * EPC;
      if (!(r < ti.rows && col < a.K)) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(tile + r * TL::ROWB + cc * 16);
      uint32_t words[EPC / 4];
      if (!quant_chunk_fast<T>(v, inv, words)) quant_chunk_exact<T>(v, inv, scale, words);
      if (static_cast<unsigned>(ti.row_start + r) >= static_cast<unsigned>(a.M)) {
        atomicOr(&g_err_quant, kErrBadIndex);  // never store outside qA
        continue;
      }
      int8_t* dst = a.qA + static_cast<int64_t>(ti.row_start + r) * a.K + col;
      if constexpr (EPC == 8) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(words[0], words[1]);
      } else {
        *reinterpret_cast<uint32_t*>(dst) = words[0];
      }
    }
    // release the stage to the producer
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&s_empty[st]));
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

int dtype_size(int dtype) { return dtype == I8MOE_FP32 ? 4 : 2; }

PFN_cuTensorMapEncodeTiled_v12000 g_encode_q = nullptr;
std::once_flag g_encode_q_once;

int encode_fn() {
  std::call_once(g_encode_q_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode_q = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode_q) return set_error(I8MOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  return I8MOE_OK;
}

// 2-D tensor map over a row-major [rows, cols] matrix with a box of
// 128 columns x box_rows rows, no swizzle, zero fill out of bounds.
int make_src_map(CUtensorMap* m, const void* base, int dtype, int64_t rows, int64_t cols,
                 int box_rows) {
  const CUtensorMapDataType dt = dtype == I8MOE_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dtype == I8MOE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * dtype_size(dtype))};
  cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode_q(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(I8MOE_ERR_CUDA, "cuTensorMapEncodeTiled(quant source) failed");
  return I8MOE_OK;
}

template <typename T, int TM, int MODE>
int launch_quant_t(const CUtensorMap& tmap, QuantArgs a, int rows_upper, cudaStream_t st) {
  using TL = QuantTile<T, TM, MODE>;
  auto kern = quant_kernel<T, TM, MODE>;
  const int smem = TL::NS * TL::STAGEB + 2 * (a.E + 1) * 4 + 1024;
  I8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, TL::THREADS, smem) !=
          cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int64_t items_upper = static_cast<int64_t>(rows_upper) * a.Kb;
  const int grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(static_cast<int64_t>(per_sm) * num_sms(current_device()), items_upper)));
  kern<<<grid, TL::THREADS, smem, st>>>(tmap, a);
  return check_launch("quant");
}

template <int MODE>
int launch_quant_mode(int dtype, int tm, const CUtensorMap& tmap, const QuantArgs& a,
                      int rows_upper, cudaStream_t st) {
  // (one CTA per SM; see quant_kernel)
  if (dtype == I8MOE_BF16) {
    return tm == 64 ? launch_quant_t<__nv_bfloat16, 64, MODE>(tmap, a, rows_upper, st)
                    : launch_quant_t<__nv_bfloat16, 128, MODE>(tmap, a, rows_upper, st);
  } else if (dtype == I8MOE_FP16) {
    return tm == 64 ? launch_quant_t<__half, 64, MODE>(tmap, a, rows_upper, st)
                    : launch_quant_t<__half, 128, MODE>(tmap, a, rows_upper, st);
  }
  return tm == 64 ? launch_quant_t<float, 64, MODE>(tmap, a, rows_upper, st)
                  : launch_quant_t<float, 128, MODE>(tmap, a, rows_upper, st);
}

// src rows/cols describe the TMA source: direct [M, K], gather [n_src, K],
// silu [M, 2K].
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
  int rc = encode_fn();
  if (rc) return rc;
  CUtensorMap tmap;
  rc = make_src_map(&tmap, src, dtype, src_rows, src_cols, mode == kGather ? 1 : static_cast<int>(tm));
  if (rc) return rc;
  QuantArgs a{};
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
  if (mode == kDirect) rc = launch_quant_mode<kDirect>(dtype, t, tmap, a, ru, st);
  else if (mode == kGather) rc = launch_quant_mode<kGather>(dtype, t, tmap, a, ru, st);
  else rc = launch_quant_mode<kSilu>(dtype, t, tmap, a, ru, st);
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
