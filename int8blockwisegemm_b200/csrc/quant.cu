// Grouped per-(expert M-tile x 128-K block) INT8 activation quantisation
// with the two-level (Q int32, F fp32) scale factorisation folded in.
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
// Launch: one thread-block cluster of C = min(8, Kb) CTAs per scale row; CTA
// rank j quantises K-blocks j, j+C, ...  Each CTA keeps its block scales in
// shared memory; after a cluster barrier every CTA reads the scales of its
// super-groups from its peers (distributed shared memory) and writes Q (and
// the first CTA of a group writes F), so neither a global scale matrix nor a
// second kernel is needed.
//
// x / scale is evaluated as x * (1/scale) first; whenever any product of a
// thread lies within 1e-4 of a rounding tie (or is not finite) the thread
// recomputes its elements with the IEEE quotient.  The product differs from
// the IEEE quotient by less than 2e-5 for |x/scale| <= 128, so the rounded
// integers are identical to round(x / scale) for every input.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

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

constexpr int kThreads = 256;
constexpr int kMaxCluster = 8;
constexpr int kMaxKbPerCta = 64;  // Kb <= 512 (K <= 65536)

enum Mode { kDirect = 0, kGather = 1, kSilu = 2 };

struct QuantArgs {
  const void* src;
  int64_t ld;      // elements per source row
  int M;           // rows of qA
  int K;           // quantised columns
  int topk;        // gather mode
  const int32_t* pidx;
  const int32_t* eo;  // [E+1]
  const int32_t* so;  // [E+1]
  int E;
  int Kb;
  int csize;
  float qmax;
  int sg;
  int nsg;
  int8_t* qA;
  int32_t* Q;
  float* F;
};

__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Low byte of the float bits of (y + 1.5*2^23) is round-to-nearest-even(y)
// as a two's-complement byte for |y| < 2^22.
__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d) {
  const uint32_t lo = __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x0040);
  const uint32_t hi = __byte_perm(__float_as_uint(c), __float_as_uint(d), 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

__device__ __forceinline__ int8_t quant_exact(float x, float scale) {
  float v = __fdiv_rn(x, scale);
  v = fminf(fmaxf(v, -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(roundf(v)));
}

template <typename T>
__device__ __forceinline__ float elem(const uint4& v, int e) {
  return Num<T>::to_f(reinterpret_cast<const T*>(&v)[e]);
}

template <typename T, int TM, int MODE>
__global__ void __launch_bounds__(kThreads) quant_kernel(QuantArgs a) {
  constexpr int EPC = 16 / sizeof(T);    // elements per 16-B chunk
  constexpr int CPR = 128 / EPC;         // chunks per 128-wide row segment
  constexpr int RPP = kThreads / CPR;    // rows per pass
  constexpr int PASSES = TM / RPP;
  static_assert(TM % RPP == 0, "tile rows");

  __shared__ float s_scale[kMaxKbPerCta];
  __shared__ float s_red[kThreads / 32];

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(blockIdx.x % a.csize);
  const int s = static_cast<int>(blockIdx.x / a.csize);
  const int total = __ldg(a.so + a.E);
  if (s >= total) return;  // the whole cluster shares s: uniform exit

  // expert owning scale row s: last e in [0, E) with so[e] <= s
  int lo = 0, hi = a.E;
  while (lo + 1 < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(a.so + mid) <= s) lo = mid; else hi = mid;
  }
  const int e = lo;
  const int row_start = __ldg(a.eo + e) + (s - __ldg(a.so + e)) * TM;
  const int row_end = min(min(__ldg(a.eo + e + 1), a.M), row_start + TM);

  const int tid = threadIdx.x;
  const int cr = tid % CPR;
  const int r0 = tid / CPR;

  // source row of every pass (gather: hidden row of the expanded row)
  int srow[PASSES];
#pragma unroll
  for (int p = 0; p < PASSES; ++p) {
    const int row = row_start + r0 + p * RPP;
    srow[p] = row < row_end ? (MODE == kGather ? __ldg(a.pidx + row) / a.topk : row) : -1;
  }
  const T* src = static_cast<const T*>(a.src);

  int nkb_local = 0;
  for (int kb = rank; kb < a.Kb; kb += a.csize, ++nkb_local) {
    const int col = kb * 128 + cr * EPC;
    const bool colok = col < a.K;
    uint4 v[PASSES];
#pragma unroll
    for (int p = 0; p < PASSES; ++p) {
      v[p] = make_uint4(0, 0, 0, 0);
      if (srow[p] >= 0 && colok) {
        const T* rp = src + static_cast<int64_t>(srow[p]) * a.ld + col;
        if (MODE == kSilu) {
          const uint4 g = __ldg(reinterpret_cast<const uint4*>(rp));
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(rp + a.K));
          T* o = reinterpret_cast<T*>(&v[p]);
#pragma unroll
          for (int i = 0; i < EPC; ++i) {
            const float gf = elem<T>(g, i);
            const float sl = __fdiv_rn(gf, 1.0f + expf(-gf));
            const float sn = Num<T>::to_f(Num<T>::from_f(sl));
            o[i] = Num<T>::from_f(sn * elem<T>(u, i));
          }
        } else {
          v[p] = __ldg(reinterpret_cast<const uint4*>(rp));
        }
      }
    }
    // tile absmax (NaN-ignoring, as tl.max / fmaxf)
    float m = 0.0f;
#pragma unroll
    for (int p = 0; p < PASSES; ++p)
#pragma unroll
      for (int i = 0; i < EPC; ++i) m = fmaxf(m, fabsf(elem<T>(v[p], i)));
    unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
    if ((tid & 31) == 0) s_red[tid >> 5] = __uint_as_float(mb);
    __syncthreads();
    float amax = s_red[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) amax = fmaxf(amax, s_red[w]);
    __syncthreads();
    const float scale = __fdiv_rn(fmaxf(amax, 1e-10f), 127.0f);
    const float inv = __frcp_rn(scale);
    if (tid == 0) s_scale[nkb_local] = scale;

    // quantise: fast product path, packed as we go
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    constexpr int WPC = EPC / 4;           // packed words per chunk
    uint32_t packed[PASSES][WPC];
    float dmax = 0.0f;
#pragma unroll
    for (int p = 0; p < PASSES; ++p)
#pragma unroll
      for (int w = 0; w < WPC; ++w) {
        float tt[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float y = __fmul_rn(elem<T>(v[p], 4 * w + i), inv);
          tt[i] = __fadd_rn(y, kMagic);
          dmax = max_nan(dmax, fabsf(y - (tt[i] - kMagic)));
        }
        packed[p][w] = pack4(tt[0], tt[1], tt[2], tt[3]);
      }
    if (!(dmax < 0.4999f)) {
      // a product lies near a rounding tie (or is not finite): exact path
#pragma unroll
      for (int p = 0; p < PASSES; ++p)
#pragma unroll
        for (int w = 0; w < WPC; ++w) {
          uint32_t word = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int8_t q = quant_exact(elem<T>(v[p], 4 * w + i), scale);
            word |= static_cast<uint32_t>(static_cast<uint8_t>(q)) << (8 * i);
          }
          packed[p][w] = word;
        }
    }
#pragma unroll
    for (int p = 0; p < PASSES; ++p) {
      if (!(srow[p] >= 0 && colok)) continue;
      const int row = row_start + r0 + p * RPP;
      int8_t* dst = a.qA + static_cast<int64_t>(row) * a.K + col;
      if constexpr (WPC == 2) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(packed[p][0], packed[p][1]);
      } else {
        *reinterpret_cast<uint32_t*>(dst) = packed[p][0];
      }
    }
  }

  // two-level scale factorisation across the cluster
  cluster.sync();
  for (int li = tid; li < nkb_local; li += kThreads) {
    const int kb = rank + li * a.csize;
    const int g = kb / a.sg;
    const int glo = g * a.sg;
    const int ghi = min(glo + a.sg, a.Kb);
    float smax = 0.0f;
    for (int k2 = glo; k2 < ghi; ++k2) {
      const float* peer = cluster.map_shared_rank(s_scale, k2 % a.csize);
      smax = fmaxf(smax, fabsf(peer[k2 / a.csize]));
    }
    const float fg = __fdiv_rn(fmaxf(smax, 1e-12f), a.qmax);
    const float qv = rintf(__fdiv_rn(s_scale[li], fg));
    a.Q[static_cast<int64_t>(s) * a.Kb + kb] = __float2int_rz(qv);
    if (kb == glo) a.F[static_cast<int64_t>(s) * a.nsg + g] = fg;
  }
  cluster.sync();
}

// Standalone Q/F factorisation of an fp32 scale matrix (one warp per row
// and super-group).
__global__ void quantize_scales_kernel(const float* __restrict__ scale, int rows, int kb,
                                       float qmax, int sg, int nsg, int32_t* Q, float* F) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows * nsg) return;
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

template <typename T, int TM, int MODE>
int launch_quant_t(const QuantArgs& a, int rows_upper, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows_upper * a.csize), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  I8_CUDA(cudaLaunchKernelEx(&cfg, quant_kernel<T, TM, MODE>, a));
  return I8MOE_OK;
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
  return tm == 64 ? launch_quant_t<float, 64, MODE>(a, rows_upper, st)
                  : launch_quant_t<float, 128, MODE>(a, rows_upper, st);
}

int launch_quant(int mode, const void* src, int dtype, int64_t ld, int64_t M, int64_t K,
                 const int32_t* pidx, int64_t topk, const int32_t* eo, int64_t E, int64_t tm,
                 int64_t block_k, int64_t q_max, int64_t sg, int8_t* qA, int32_t* Q, float* F,
                 int32_t* so, int so_ready, cudaStream_t st) {
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16 || dtype == I8MOE_FP32,
             "quant: A must be float32, float16 or bfloat16");
  I8_REQUIRE(block_k == 128, "quant: block_k must be 128 (the only quant block the GEMM reads)");
  I8_REQUIRE(tm == 64 || tm == 128, "quant: tile_m must be 64 or 128");
  I8_REQUIRE(sg > 0 && q_max > 0, "quant: super_group_size and q_max must be positive");
  I8_REQUIRE(E >= 1 && E <= 65536, "quant: expert_offsets must have 2..65537 entries");
  I8_REQUIRE(K % 8 == 0, "quant: K must be a multiple of 8");
  I8_REQUIRE(M >= 0 && M < (int64_t(1) << 31), "quant: bad M");
  const int64_t Kb = (K + block_k - 1) / block_k;
  const int csize = static_cast<int>(std::min<int64_t>(kMaxCluster, std::max<int64_t>(Kb, 1)));
  I8_REQUIRE((Kb + csize - 1) / csize <= kMaxKbPerCta, "quant: K too large (max 65536)");
  const uintptr_t al = reinterpret_cast<uintptr_t>(src) | static_cast<uintptr_t>(ld * dtype_size(dtype));
  I8_REQUIRE(al % 16 == 0, "quant: source rows must be 16-byte aligned");
  I8_REQUIRE(reinterpret_cast<uintptr_t>(qA) % 8 == 0, "quant: qA must be 8-byte aligned");
  if (!so_ready) {
    scale_offsets_kernel<<<1, 1024, 0, st>>>(eo, static_cast<int>(E), static_cast<int>(tm), so);
    int rc = check_launch("scale_offsets");
    if (rc) return rc;
  }
  const int64_t rows_upper = (M + tm - 1) / tm + E;
  if (M == 0 || K == 0) return I8MOE_OK;
  QuantArgs a{};
  a.src = src;
  a.ld = ld;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.topk = static_cast<int>(topk);
  a.pidx = pidx;
  a.eo = eo;
  a.so = so;
  a.E = static_cast<int>(E);
  a.Kb = static_cast<int>(Kb);
  a.csize = csize;
  a.qmax = static_cast<float>(q_max);
  a.sg = static_cast<int>(sg);
  a.nsg = static_cast<int>((Kb + sg - 1) / sg);
  a.qA = qA;
  a.Q = Q;
  a.F = F;
  const int ru = static_cast<int>(rows_upper);
  const int t = static_cast<int>(tm);
  int rc;
  if (mode == kDirect) rc = launch_quant_mode<kDirect>(dtype, t, a, ru, st);
  else if (mode == kGather) rc = launch_quant_mode<kGather>(dtype, t, a, ru, st);
  else rc = launch_quant_mode<kSilu>(dtype, t, a, ru, st);
  if (rc) return rc;
  return check_launch("quant");
}

}  // namespace
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
  return launch_quant(kDirect, A, dtype, K, M, K, nullptr, 1, expert_offsets, n_expert, tile_m,
                      block_k, q_max, super_group_size, qA, Q, F, scale_offsets,
                      scale_offsets_ready, static_cast<cudaStream_t>(stream));
}

int i8moe_quant_permute(const void* hidden, int dtype, int64_t n_token, int64_t K,
                        const int32_t* permuted_idx, int64_t M, int64_t topk,
                        const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                        int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                        int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                        i8moe_stream_t stream) {
  (void)n_token;
  I8_REQUIRE(topk > 0, "quant_permute: topk must be positive");
  return launch_quant(kGather, hidden, dtype, K, M, K, permuted_idx, topk, expert_offsets,
                      n_expert, tile_m, block_k, q_max, super_group_size, qA, Q, F,
                      scale_offsets, scale_offsets_ready, static_cast<cudaStream_t>(stream));
}

int i8moe_quant_silu(const void* mm1, int dtype, int64_t M, int64_t N,
                     const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                     int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                     int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                     i8moe_stream_t stream) {
  return launch_quant(kSilu, mm1, dtype, 2 * N, M, N, nullptr, 1, expert_offsets, n_expert,
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
  quantize_scales_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      scale, static_cast<int>(rows), static_cast<int>(kb), static_cast<float>(q_max),
      static_cast<int>(super_group_size), static_cast<int>(nsg), Q, F);
  return check_launch("quantize_scales");
}

}  // extern "C"
