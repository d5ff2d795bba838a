// Routing (stable counting sort of expanded rows by expert), row gather,
// top-k weighted unpermute and silu_and_mul for sm_100a.
//
// Routing replaces the reference's CUB radix sort + binary-search offsets +
// permutation-map kernels (csrc/permute_unpermute_kernels/
// moe_permute_unpermute_kernel.cu:25-169, .inl:3-118) by three small
// kernels over chunks of 2048 keys:
//   route_hist    -- per-chunk bucket histogram (bucket = key's low
//                    experts_to_bits(n_expert) bits, the bits CUB sorts on)
//   route_scan    -- one CTA: per-bucket exclusive scan across chunks and
//                    across buckets; writes expert_first_token_offset (and,
//                    for the fused forward, int32 offsets, problem sizes and
//                    quant scale offsets)
//   route_scatter -- stable rank of every key inside its chunk
//                    (warp match_any + per-warp counts), destination =
//                    chunk bucket base + rank; writes inv/permuted maps.
// A stable counting sort on the same bits yields exactly the order of the
// stable LSD radix sort, so the maps are bit-identical.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace i8moe {

static __device__ unsigned g_err_route;

int read_route_error(uint32_t* w, int clear) {
  unsigned v = 0;
  I8_CUDA(cudaMemcpyFromSymbol(&v, g_err_route, sizeof(v)));
  if (clear) {
    unsigned z = 0;
    I8_CUDA(cudaMemcpyToSymbol(g_err_route, &z, sizeof(z)));
  }
  *w = v;
  return I8MOE_OK;
}

namespace {

constexpr int kThreads = 256;
constexpr int kKeysPerThread = 8;
constexpr int kChunk = kThreads * kKeysPerThread;  // 2048 keys per chunk
constexpr int kMaxBuckets = 4096;                  // n_expert <= 2048

int experts_to_bits(int64_t n_expert) {
  // floor(log2(2E - 1)) + 1 == bit length of (2E - 1)
  int64_t v = 2 * n_expert - 1;
  int bits = 0;
  while (v > 0) {
    ++bits;
    v >>= 1;
  }
  return bits;
}

struct RouteArgs {
  const int32_t* ids;
  const int32_t* values;  // token_expert_indices
  const int32_t* emap;    // nullable
  int n_expert;
  int n_local;
  int R;
  int nb;  // buckets = 2^bits
  int chunks;
  int* hist;  // [chunks][nb]
  int64_t* eft;
  int32_t* inv;
  int32_t* pidx;
  // fused-forward extras (nullable)
  int32_t* eo32;
  int32_t* ps1;
  int32_t* ps2;
  int32_t* so;
  int n_out1, k1, n_out2, k2, tile_m;
};

// Sort key of an expert id: the (local) expert, or key + n_expert for ids
// mapped to no local expert, keeping the bits the reference's CUB sort uses.
__device__ __forceinline__ int route_key_of(const RouteArgs& a, int key) {
  if (a.emap != nullptr) {
    if (key < 0 || key >= a.n_expert) {
      atomicOr(&g_err_route, kErrBadIndex);
      key = key + a.n_expert;
    } else {
      const int local = __ldg(a.emap + key);
      key = (local == -1) ? key + a.n_expert : local;
    }
  }
  return key & (a.nb - 1);
}

__device__ __forceinline__ int route_key(const RouteArgs& a, int i) {
  return route_key_of(a, __ldg(a.ids + i));
}

__global__ void __launch_bounds__(kThreads) route_hist(RouteArgs a) {
  extern __shared__ int s_hist[];
  for (int b = threadIdx.x; b < a.nb; b += kThreads) s_hist[b] = 0;
  __syncthreads();
  const int base = blockIdx.x * kChunk;
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    const int i = base + j * kThreads + threadIdx.x;
    if (i < a.R) atomicAdd(&s_hist[route_key(a, i)], 1);
  }
  __syncthreads();
  int* out = a.hist + static_cast<int64_t>(blockIdx.x) * a.nb;
  for (int b = threadIdx.x; b < a.nb; b += kThreads) out[b] = s_hist[b];
}

// ---------------------------------------------------------------------------
// Router: top-k over biased logits, softmax over the selected logits
// ---------------------------------------------------------------------------
// One warp per token; lane l holds logits l, l+32, ...  k rounds of warp
// arg-max pick the experts (ties to the lower expert id) by logit + bias; the
// weights are the softmax of the selected unbiased logits (renormalised over
// the top-k), as the benchmark's seeded router builds them.  With
// `a.hist != nullptr` the CTA also writes the routing histogram of its key
// chunk (the route_hist output), so routing can start from the logits.
struct RouterArgs {
  const float* logits;  // [T, E]
  const float* bias;    // [E] or null
  int T, E, k;
  int32_t* ids;         // [T, k]
  float* weights;       // [T, k]
};

// Returns the expert picked in round `lane` (lanes 0..k-1).
template <int VPL>
__device__ __forceinline__ int router_token(const RouterArgs& r, int t, int lane) {
  const float* row = r.logits + static_cast<int64_t>(t) * r.E;
  float v[VPL], sv[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < r.E ? __ldg(row + e) : 0.f;
    sv[i] = e < r.E ? v[i] + (r.bias ? __ldg(r.bias + e) : 0.f) : -INFINITY;
  }
  unsigned taken = 0u;
  int my_id = 0;
  float my_logit = -INFINITY;
  for (int j = 0; j < r.k; ++j) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (!(taken >> i & 1u) && e < r.E && (sv[i] > bv || be == 0x7fffffff)) {
        bv = sv[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    // the owner marks it and broadcasts the unbiased logit
    float lg = 0.f;
    if ((be & 31) == lane) {
      const int i = be >> 5;
#pragma unroll
      for (int q = 0; q < VPL; ++q)
        if (q == i) {
          taken |= 1u << q;
          lg = v[q];
        }
    }
    lg = __shfl_sync(0xffffffffu, lg, be & 31);
    if (lane == j) {
      my_id = be;
      my_logit = lg;
    }
  }
  // softmax over the k selected logits (lanes 0..k-1)
  float m = lane < r.k ? my_logit : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float ex = lane < r.k ? expf(my_logit - m) : 0.f;
  float sum = ex;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane < r.k) {
    r.ids[static_cast<int64_t>(t) * r.k + lane] = my_id;
    r.weights[static_cast<int64_t>(t) * r.k + lane] = __fdiv_rn(ex, sum);
  }
  return my_id;
}

template <int VPL>
__global__ void __launch_bounds__(kThreads) router_kernel(RouterArgs r, RouteArgs a) {
  extern __shared__ int s_hist[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (a.hist == nullptr) {
    const int t = blockIdx.x * (kThreads / 32) + warp;
    if (t < r.T) router_token<VPL>(r, t, lane);
    return;
  }
  // fused with route_hist: this CTA owns keys [c*kChunk, (c+1)*kChunk)
  for (int b = threadIdx.x; b < a.nb; b += kThreads) s_hist[b] = 0;
  __syncthreads();
  const int key0 = blockIdx.x * kChunk;
  const int key1 = min(key0 + kChunk, a.R);
  const int t0 = key0 / r.k, t1 = (key1 + r.k - 1) / r.k;
  for (int t = t0 + warp; t < t1; t += kThreads / 32) {
    // a token straddling two chunks is routed by both CTAs, identically
    const int id = router_token<VPL>(r, t, lane);
    if (lane < r.k) {
      const int i = t * r.k + lane;
      if (i >= key0 && i < key1) atomicAdd(&s_hist[route_key_of(a, id)], 1);
    }
  }
  __syncthreads();
  int* out = a.hist + static_cast<int64_t>(blockIdx.x) * a.nb;
  for (int b = threadIdx.x; b < a.nb; b += kThreads) out[b] = s_hist[b];
}

// Single CTA of 1024 threads.
__global__ void __launch_bounds__(1024) route_scan(RouteArgs a) {
  __shared__ int s_tot[kMaxBuckets];
  __shared__ int s_warp[32];
  const int tid = threadIdx.x;
  // 1) per-bucket exclusive scan across chunks (in place), bucket totals.
  for (int b = tid; b < a.nb; b += 1024) {
    int run = 0;
    int c = 0;
    for (; c + 16 <= a.chunks; c += 16) {  // 16 loads in flight per thread
      int v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) v[u] = a.hist[static_cast<int64_t>(c + u) * a.nb + b];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        a.hist[static_cast<int64_t>(c + u) * a.nb + b] = run;
        run += v[u];
      }
    }
    for (; c < a.chunks; ++c) {
      const int v = a.hist[static_cast<int64_t>(c) * a.nb + b];
      a.hist[static_cast<int64_t>(c) * a.nb + b] = run;
      run += v;
    }
    s_tot[b] = run;
  }
  __syncthreads();
  // 2) exclusive scan of the totals over buckets (contiguous segments).
  const int per = (a.nb + 1023) / 1024;
  const int lo = tid * per;
  int local = 0;
  for (int i = 0; i < per; ++i)
    if (lo + i < a.nb) local += s_tot[lo + i];
  const int lane = tid & 31, warp = tid >> 5;
  int v = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) s_warp[warp] = v;
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
  int prefix = v - local + (warp > 0 ? s_warp[warp - 1] : 0);
  for (int i = 0; i < per; ++i) {
    if (lo + i < a.nb) {
      const int t = s_tot[lo + i];
      s_tot[lo + i] = prefix;
      prefix += t;
    }
  }
  __syncthreads();
  // 3) chunk bases become absolute destinations (8 loads in flight per
  // thread before the stores, not one round trip per entry).
  {
    const int total = a.chunks * a.nb;
    for (int i0 = tid; i0 < total; i0 += 8 * 1024) {
      int v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i0 + 1024 * u < total) v[u] = a.hist[i0 + 1024 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i0 + 1024 * u < total) a.hist[i0 + 1024 * u] = v[u] + s_tot[(i0 + 1024 * u) % a.nb];
    }
  }
  // 4) expert offsets (n_local < nb always).
  for (int e = tid; e <= a.n_local; e += 1024) {
    const int off = s_tot[e];
    a.eft[e] = off;
    if (a.eo32) a.eo32[e] = off;
  }
  if (a.ps1 != nullptr) {
    for (int e = tid; e < a.n_local; e += 1024) {
      const int cnt = s_tot[e + 1] - s_tot[e];
      a.ps1[3 * e + 0] = cnt;
      a.ps1[3 * e + 1] = a.n_out1;
      a.ps1[3 * e + 2] = a.k1;
      a.ps2[3 * e + 0] = cnt;
      a.ps2[3 * e + 1] = a.n_out2;
      a.ps2[3 * e + 2] = a.k2;
    }
  }
  if (a.so != nullptr) {
    // exclusive cumsum of ceil(count_e / tile_m); reuse the scan scheme.
    __syncthreads();
    const int E = a.n_local;
    const int per2 = (E + 1023) / 1024;
    const int lo2 = tid * per2;
    int loc = 0;
    for (int i = 0; i < per2; ++i)
      if (lo2 + i < E) loc += (s_tot[lo2 + i + 1] - s_tot[lo2 + i] + a.tile_m - 1) / a.tile_m;
    int x = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    __syncthreads();
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
    for (int i = 0; i < per2; ++i) {
      if (lo2 + i < E) {
        a.so[lo2 + i] = pre;
        pre += (s_tot[lo2 + i + 1] - s_tot[lo2 + i] + a.tile_m - 1) / a.tile_m;
      }
    }
    if (lo2 < E && lo2 + per2 >= E) a.so[E] = pre;
    if (E == 0 && tid == 0) a.so[0] = 0;
  }
}

// Stable scatter.  Dynamic smem: running[nb] + wcnt[8][nb].
__global__ void __launch_bounds__(kThreads) route_scatter(RouteArgs a, int check_limit) {
  extern __shared__ int s_mem[];
  int* running = s_mem;
  int* wcnt = s_mem + a.nb;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int* base = a.hist + static_cast<int64_t>(blockIdx.x) * a.nb;
  for (int b = tid; b < a.nb; b += kThreads) running[b] = base[b];
  for (int i = tid; i < 8 * a.nb; i += kThreads) wcnt[i] = 0;
  const int limit = check_limit ? static_cast<int>(a.eft[a.n_local]) : a.R;
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int j = 0; j < kKeysPerThread; ++j) {
    const int i = blockIdx.x * kChunk + j * kThreads + tid;
    const bool valid = i < a.R;
    const int b = valid ? route_key(a, i) : a.nb;  // invalid lanes form their own group
    const unsigned m = __match_any_sync(0xffffffffu, b);
    const int rank = __popc(m & lt_mask);
    const int cnt = __popc(m);
    const bool leader = (m & lt_mask) == 0;
    if (valid && leader) wcnt[warp * a.nb + b] = cnt;
    __syncthreads();
    int dest = 0;
    if (valid) {
      dest = running[b] + rank;
      for (int w = 0; w < warp; ++w) dest += wcnt[w * a.nb + b];
    }
    __syncthreads();
    if (valid && leader) {
      atomicAdd(&running[b], cnt);
      wcnt[warp * a.nb + b] = 0;
    }
    if (valid) {
      // token_expert_indices is arange in the reference; null means exactly that
      const int value = a.values != nullptr ? __ldg(a.values + i) : i;
      if (value >= 0 && value < a.R) {
        a.inv[value] = dest;
      } else {
        atomicOr(&g_err_route, kErrBadIndex);
      }
      // every slot is written once: the row, or past the local experts' rows
      // the sentinel n_token * topk the reference pre-fills permuted_idx with
      a.pidx[dest] = dest < limit ? value : a.R;
    }
    __syncthreads();
  }
}

template <int VEC_BYTES>
__global__ void expand_rows(const uint4* __restrict__ in, uint4* __restrict__ out,
                            const int32_t* __restrict__ pidx, const int64_t* eft, int n_local,
                            int R, int topk, int vecs_per_row, int check_limit) {
  const int limit = check_limit ? static_cast<int>(eft[n_local]) : R;
  for (int d = blockIdx.x; d < limit; d += gridDim.x) {
    const int src_row = __ldg(pidx + d) / topk;
    const uint4* s = in + static_cast<int64_t>(src_row) * vecs_per_row;
    uint4* o = out + static_cast<int64_t>(d) * vecs_per_row;
    for (int v = threadIdx.x; v < vecs_per_row; v += blockDim.x) o[v] = __ldg(s + v);
  }
}

// out[t] = dtype(sum_j fma(w[t,j], x[inv[t,j]], acc)), fp32 accumulation in
// j order (finalizeMoeRoutingKernel, .inl:132-188).  Two tokens per CTA:
// both tokens' inverse indices, then all their rows, are in flight together
// (one token per CTA measured 66.8 against 63.5 us at the default shape).
template <typename T>
__global__ void __launch_bounds__(256) unpermute_kernel(const T* __restrict__ x,
                                                        const float* __restrict__ w,
                                                        const int32_t* __restrict__ inv,
                                                        const int64_t* eft, int n_local, int topk,
                                                        int vecs_per_row, T* __restrict__ out,
                                                        int n_token) {
  constexpr int EPV = 16 / sizeof(T);
  constexpr int G = 8;    // source rows in flight per token
  constexpr int TPC = 2;  // tokens per CTA
  const int t0 = blockIdx.x * TPC;
  const int64_t valid = eft ? eft[n_local] : INT64_MAX;
  for (int v = threadIdx.x; v < vecs_per_row; v += blockDim.x) {
    float acc[TPC][EPV];
#pragma unroll
    for (int tt = 0; tt < TPC; ++tt)
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[tt][e] = 0.f;
    for (int j0 = 0; j0 < topk; j0 += G) {
      uint4 raw[TPC][G];
      int idx[TPC][G];
#pragma unroll
      for (int tt = 0; tt < TPC; ++tt)
#pragma unroll
        for (int j = 0; j < G; ++j)
          idx[tt][j] = (t0 + tt < n_token && j0 + j < topk)
                           ? __ldg(inv + static_cast<int64_t>(t0 + tt) * topk + j0 + j)
                           : -1;
#pragma unroll
      for (int tt = 0; tt < TPC; ++tt)
#pragma unroll
        for (int j = 0; j < G; ++j)
          if (idx[tt][j] >= 0 && idx[tt][j] < valid)
            raw[tt][j] = __ldg(reinterpret_cast<const uint4*>(x) +
                               static_cast<int64_t>(idx[tt][j]) * vecs_per_row + v);
#pragma unroll
      for (int tt = 0; tt < TPC; ++tt)
#pragma unroll
        for (int j = 0; j < G; ++j) {
          if (idx[tt][j] >= 0 && idx[tt][j] < valid) {
            const float wt = __ldg(w + static_cast<int64_t>(t0 + tt) * topk + j0 + j);
            const T* e8 = reinterpret_cast<const T*>(&raw[tt][j]);
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[tt][e] = fmaf(wt, Num<T>::to_f(e8[e]), acc[tt][e]);
          }
        }
    }
#pragma unroll
    for (int tt = 0; tt < TPC; ++tt) {
      if (t0 + tt >= n_token) break;
      uint4 o;
      T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int e = 0; e < EPV; ++e) ov[e] = Num<T>::from_f(acc[tt][e]);
      reinterpret_cast<uint4*>(out)[static_cast<int64_t>(t0 + tt) * vecs_per_row + v] = o;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) unpermute_kernel(const T* __restrict__ x,
                                                        const float* __restrict__ w,
                                                        const int32_t* __restrict__ inv,
                                                        const int64_t* eft, int n_local, int topk,
                                                        int vecs_per_row, T* __restrict__ out) {
  constexpr int EPV = 16 / sizeof(T);
  constexpr int G = 8;  // source rows in flight per thread
  const int t = blockIdx.x;
  const int64_t valid = eft ? eft[n_local] : INT64_MAX;
  const int32_t* inv_t = inv + static_cast<int64_t>(t) * topk;
  const float* w_t = w + static_cast<int64_t>(t) * topk;
  for (int v = threadIdx.x; v < vecs_per_row; v += blockDim.x) {
    float acc[EPV];
#pragma unroll
    for (int e = 0; e < EPV; ++e) acc[e] = 0.f;
    for (int j0 = 0; j0 < topk; j0 += G) {
      uint4 raw[G];
      int idx[G];
#pragma unroll
      for (int j = 0; j < G; ++j) {
        idx[j] = (j0 + j < topk) ? __ldg(inv_t + j0 + j) : -1;
        if (idx[j] >= 0 && idx[j] < valid)
          raw[j] = __ldg(reinterpret_cast<const uint4*>(x) +
                         static_cast<int64_t>(idx[j]) * vecs_per_row + v);
      }
#pragma unroll
      for (int j = 0; j < G; ++j) {
        if (idx[j] >= 0 && idx[j] < valid) {
          const float wt = __ldg(w_t + j0 + j);
          const T* e8 = reinterpret_cast<const T*>(&raw[j]);
#pragma unroll
          for (int e = 0; e < EPV; ++e) acc[e] = fmaf(wt, Num<T>::to_f(e8[e]), acc[e]);
        }
      }
    }
    uint4 o;
    T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int e = 0; e < EPV; ++e) ov[e] = Num<T>::from_f(acc[e]);
    reinterpret_cast<uint4*>(out)[static_cast<int64_t>(t) * vecs_per_row + v] = o;
  }
}

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t rows,
                                int d) {
  constexpr int EPV = 16 / sizeof(T);
  const int vpr = d / EPV;
  const int64_t total = rows * vpr;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vpr;
    const int c = static_cast<int>(i - r * vpr);
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(in + r * 2 * d) + c);
    const uint4 uv = __ldg(reinterpret_cast<const uint4*>(in + r * 2 * d + d) + c);
    const T* g8 = reinterpret_cast<const T*>(&gv);
    const T* u8 = reinterpret_cast<const T*>(&uv);
    uint4 o;
    T* o8 = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      const float g = Num<T>::to_f(g8[e]);
      const float s = __fdiv_rn(g, 1.0f + expf(-g));
      const float sn = Num<T>::to_f(Num<T>::from_f(s));
      o8[e] = Num<T>::from_f(sn * Num<T>::to_f(u8[e]));
    }
    reinterpret_cast<uint4*>(out + r * d)[c] = o;
  }
}

size_t route_ws_bytes(int64_t R, int64_t n_expert) {
  const int64_t nb = int64_t(1) << experts_to_bits(n_expert);
  const int64_t chunks = std::max<int64_t>(1, (R + kChunk - 1) / kChunk);
  return static_cast<size_t>(chunks * nb * sizeof(int));
}

struct FusedExtras {
  int32_t* eo32 = nullptr;
  int32_t* ps1 = nullptr;
  int32_t* ps2 = nullptr;
  int32_t* so = nullptr;
  int n_out1 = 0, k1 = 0, n_out2 = 0, k2 = 0, tile_m = 128;
};

int router_vpl(int64_t E) { return E <= 256 ? 8 : (E <= 512 ? 16 : (E <= 1024 ? 32 : 0)); }

// r != nullptr: the first routing kernel is the router (top-k + softmax from
// logits), which writes topk_ids/weights and the chunk histogram.
int launch_route(const int32_t* topk_ids, const int32_t* tei, const int32_t* emap,
                 int64_t n_token, int64_t topk, int64_t n_expert, int64_t n_local, int64_t* eft,
                 int32_t* inv, int32_t* pidx, void* ws, size_t ws_bytes, cudaStream_t st,
                 const FusedExtras& fx, const RouterArgs* router = nullptr) {
  I8_REQUIRE(n_token >= 0 && topk > 0, "moe_permute: bad n_token/topk");
  I8_REQUIRE(n_expert >= 1 && n_expert <= 2048, "moe_permute: n_expert must be in [1, 2048]");
  I8_REQUIRE(n_local >= 0 && n_local <= n_expert,
             "expert_first_token_offset shape != n_local_expert+1");
  const int64_t R = n_token * topk;
  I8_REQUIRE(R < (int64_t(1) << 31) - 1, "moe_permute: too many rows");
  const int bits = experts_to_bits(n_expert);
  const int nb = 1 << bits;
  const int chunks = static_cast<int>(std::max<int64_t>(1, (R + kChunk - 1) / kChunk));
  I8_REQUIRE(ws != nullptr && ws_bytes >= route_ws_bytes(R, n_expert),
             "[route] The allocated workspace is too small to run this problem.");
  RouteArgs a{};
  a.ids = topk_ids;
  a.values = tei;
  a.emap = emap;
  a.n_expert = static_cast<int>(n_expert);
  a.n_local = static_cast<int>(n_local);
  a.R = static_cast<int>(R);
  a.nb = nb;
  a.chunks = chunks;
  a.hist = static_cast<int*>(ws);
  a.eft = eft;
  a.inv = inv;
  a.pidx = pidx;
  a.eo32 = fx.eo32;
  a.ps1 = fx.ps1;
  a.ps2 = fx.ps2;
  a.so = fx.so;
  a.n_out1 = fx.n_out1;
  a.k1 = fx.k1;
  a.n_out2 = fx.n_out2;
  a.k2 = fx.k2;
  a.tile_m = fx.tile_m;
  const size_t smem_hist = nb * sizeof(int);
  const size_t smem_scatter = 9 * nb * sizeof(int);
  if (smem_scatter > 48 * 1024) {
    I8_CUDA(cudaFuncSetAttribute(route_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem_scatter)));
  }
  if (router != nullptr) {
    const int vpl = router_vpl(router->E);
    if (vpl == 8) router_kernel<8><<<chunks, kThreads, smem_hist, st>>>(*router, a);
    else if (vpl == 16) router_kernel<16><<<chunks, kThreads, smem_hist, st>>>(*router, a);
    else router_kernel<32><<<chunks, kThreads, smem_hist, st>>>(*router, a);
  } else {
    route_hist<<<chunks, kThreads, smem_hist, st>>>(a);
  }
  route_scan<<<1, 1024, 0, st>>>(a);
  route_scatter<<<chunks, kThreads, smem_scatter, st>>>(a, emap != nullptr ? 1 : 0);
  return check_launch("route kernels");
}

}  // namespace

int launch_route_fused(const int32_t* topk_ids, const int32_t* tei, const int32_t* emap,
                       int64_t n_token, int64_t topk, int64_t n_expert, int64_t n_local,
                       int64_t* eft, int32_t* inv, int32_t* pidx, void* ws, size_t ws_bytes,
                       cudaStream_t st, int32_t* eo32, int32_t* ps1, int32_t* ps2, int32_t* so,
                       int n_out1, int k1, int n_out2, int k2, int tile_m) {
  FusedExtras fx;
  fx.eo32 = eo32;
  fx.ps1 = ps1;
  fx.ps2 = ps2;
  fx.so = so;
  fx.n_out1 = n_out1;
  fx.k1 = k1;
  fx.n_out2 = n_out2;
  fx.k2 = k2;
  fx.tile_m = tile_m;
  return launch_route(topk_ids, tei, emap, n_token, topk, n_expert, n_local, eft, inv, pidx, ws,
                      ws_bytes, st, fx);
}

// ---------------------------------------------------------------------------
// Allocation-free routing scratch
// ---------------------------------------------------------------------------
// Some callers cannot hand the routing kernels a workspace: they run without a
// caching allocator, inside a pre-sized arena, or in a loop where allocating
// device memory per call is not allowed.  For them the per-chunk histogram
// lives in a fixed device array compiled into this library.  Its size caps the
// problem (buckets x 2048-key chunks x 4 bytes); anything larger must use the
// workspace entry point.  The histogram kernel writes every slot it later
// reads, so nothing in the array has to start at zero.  There is one array per
// device, so two calls that overlap on one device (two streams, two threads)
// would race on it: calls on a device must be serialised.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB
static __device__ __align__(256) unsigned char g_route_scratch[kNoAllocScratchBytes];

constexpr int kMaxScratchDevices = 64;
struct ScratchSlot {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t status = cudaSuccess;
};
ScratchSlot g_scratch_slots[kMaxScratchDevices];

// Device address of g_route_scratch on the current device, looked up once per
// device (with that device current) and cached.
int route_scratch_ptr(void** out) {
  int dev = -1;
  I8_CUDA(cudaGetDevice(&dev));
  I8_REQUIRE(dev >= 0 && dev < kMaxScratchDevices,
             "moe_permute_metadata_noalloc: device ordinal %d out of range", dev);
  ScratchSlot& slot = g_scratch_slots[dev];
  std::call_once(slot.once, [&slot] {
    void* p = nullptr;
    slot.status = cudaGetSymbolAddress(&p, g_route_scratch);
    if (slot.status == cudaSuccess) slot.ptr = p;
  });
  if (slot.status != cudaSuccess)
    return set_error(I8MOE_ERR_CUDA, std::string("cudaGetSymbolAddress(route scratch): ") +
                                         cudaGetErrorString(slot.status));
  *out = slot.ptr;
  return I8MOE_OK;
}

}  // namespace

int launch_route_noalloc(const int32_t* topk_ids, const int32_t* tei, const int32_t* emap,
                         int64_t n_token, int64_t topk, int64_t n_expert, int64_t n_local,
                         int64_t* eft, int32_t* inv, int32_t* pidx, cudaStream_t st) {
  I8_REQUIRE(n_token >= 0 && topk > 0, "moe_permute: bad n_token/topk");
  I8_REQUIRE(n_expert >= 1 && n_expert <= 2048, "moe_permute: n_expert must be in [1, 2048]");
  // bound the row count before forming it, so n_token * topk cannot overflow
  I8_REQUIRE(n_token <= INT32_MAX / topk, "moe_permute: n_token * topk must fit in int32");
  const size_t need = route_ws_bytes(n_token * topk, n_expert);
  I8_REQUIRE(need <= kNoAllocScratchBytes,
             "moe_permute_metadata_noalloc: %lld rows of %lld experts need %zu bytes of routing "
             "scratch, more than the fixed %zu-byte device buffer; use "
             "i8moe_moe_permute_metadata with a caller workspace",
             static_cast<long long>(n_token * topk), static_cast<long long>(n_expert), need,
             kNoAllocScratchBytes);
  void* ws = nullptr;
  const int rc = route_scratch_ptr(&ws);
  if (rc) return rc;
  return launch_route(topk_ids, tei, emap, n_token, topk, n_expert, n_local, eft, inv, pidx, ws,
                      kNoAllocScratchBytes, st, FusedExtras{});
}

}  // namespace i8moe

using namespace i8moe;

static int dtype_size(int dtype) { return dtype == I8MOE_FP32 ? 4 : 2; }

extern "C" {

size_t i8moe_route_workspace_size(int64_t n_rows, int64_t n_expert) {
  if (n_expert < 1) return 0;
  return route_ws_bytes(n_rows, n_expert);
}

int i8moe_moe_permute_metadata(const int32_t* topk_ids, const int32_t* token_expert_indices,
                               const int32_t* expert_map, int64_t n_token, int64_t topk,
                               int64_t n_expert, int64_t n_local_expert,
                               int64_t* expert_first_token_offset, int32_t* inv_permuted_idx,
                               int32_t* permuted_idx, void* workspace, size_t workspace_bytes,
                               i8moe_stream_t stream) {
  return launch_route(topk_ids, token_expert_indices, expert_map, n_token, topk, n_expert,
                      n_local_expert, expert_first_token_offset, inv_permuted_idx, permuted_idx,
                      workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                      FusedExtras{});
}

int i8moe_moe_permute_metadata_noalloc(const int32_t* topk_ids,
                                       const int32_t* token_expert_indices,
                                       const int32_t* expert_map, int64_t n_token, int64_t topk,
                                       int64_t n_expert, int64_t n_local_expert,
                                       int64_t* expert_first_token_offset,
                                       int32_t* inv_permuted_idx, int32_t* permuted_idx,
                                       i8moe_stream_t stream) {
  return launch_route_noalloc(topk_ids, token_expert_indices, expert_map, n_token, topk, n_expert,
                              n_local_expert, expert_first_token_offset, inv_permuted_idx,
                              permuted_idx, static_cast<cudaStream_t>(stream));
}

int i8moe_router_topk(const float* logits, const float* bias, int64_t n_token, int64_t n_expert,
                      int64_t topk, int32_t* topk_ids, float* topk_weights,
                      i8moe_stream_t stream) {
  I8_REQUIRE(n_token >= 0 && n_token < (int64_t(1) << 31), "router: bad n_token");
  I8_REQUIRE(router_vpl(n_expert) > 0, "router: n_expert must be in [1, 1024]");
  I8_REQUIRE(topk >= 1 && topk <= 32 && topk <= n_expert, "router: topk must be in [1, min(32, E)]");
  if (n_token == 0) return I8MOE_OK;
  RouterArgs r{logits, bias, static_cast<int>(n_token), static_cast<int>(n_expert),
               static_cast<int>(topk), topk_ids, topk_weights};
  RouteArgs a{};  // a.hist == nullptr: router only
  const unsigned grid = static_cast<unsigned>((n_token + kThreads / 32 - 1) / (kThreads / 32));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vpl = router_vpl(n_expert);
  if (vpl == 8) router_kernel<8><<<grid, kThreads, 0, st>>>(r, a);
  else if (vpl == 16) router_kernel<16><<<grid, kThreads, 0, st>>>(r, a);
  else router_kernel<32><<<grid, kThreads, 0, st>>>(r, a);
  return check_launch("router");
}

int i8moe_router_route_for_gemm(const float* logits, const float* bias, int64_t n_token,
                                int64_t n_expert, int64_t topk, int32_t* topk_ids,
                                float* topk_weights, const int32_t* token_expert_indices,
                                const int32_t* expert_map, int64_t n_local_expert,
                                int64_t* expert_first_token_offset, int32_t* inv_permuted_idx,
                                int32_t* permuted_idx, int32_t* expert_offsets,
                                int32_t* problem_sizes13, int32_t* problem_sizes2,
                                int32_t* scale_offsets, int64_t n_out1, int64_t k1,
                                int64_t n_out2, int64_t k2, int64_t tile_m, void* workspace,
                                size_t workspace_bytes, i8moe_stream_t stream) {
  I8_REQUIRE(router_vpl(n_expert) > 0, "router: n_expert must be in [1, 1024]");
  I8_REQUIRE(topk >= 1 && topk <= 32 && topk <= n_expert, "router: topk must be in [1, min(32, E)]");
  I8_REQUIRE(tile_m > 0, "route_for_gemm: tile_m must be positive");
  I8_REQUIRE(expert_offsets && problem_sizes13 && problem_sizes2 && scale_offsets,
             "route_for_gemm: every output must be given");
  RouterArgs r{logits, bias, static_cast<int>(n_token), static_cast<int>(n_expert),
               static_cast<int>(topk), topk_ids, topk_weights};
  FusedExtras fx;
  fx.eo32 = expert_offsets;
  fx.ps1 = problem_sizes13;
  fx.ps2 = problem_sizes2;
  fx.so = scale_offsets;
  fx.n_out1 = static_cast<int>(n_out1);
  fx.k1 = static_cast<int>(k1);
  fx.n_out2 = static_cast<int>(n_out2);
  fx.k2 = static_cast<int>(k2);
  fx.tile_m = static_cast<int>(tile_m);
  return launch_route(topk_ids, token_expert_indices, expert_map, n_token, topk, n_expert,
                      n_local_expert, expert_first_token_offset, inv_permuted_idx, permuted_idx,
                      workspace, workspace_bytes, static_cast<cudaStream_t>(stream), fx, &r);
}

int i8moe_moe_route_for_gemm(const int32_t* topk_ids, const int32_t* token_expert_indices,
                             const int32_t* expert_map, int64_t n_token, int64_t topk,
                             int64_t n_expert, int64_t n_local_expert,
                             int64_t* expert_first_token_offset, int32_t* inv_permuted_idx,
                             int32_t* permuted_idx, int32_t* expert_offsets,
                             int32_t* problem_sizes13, int32_t* problem_sizes2,
                             int32_t* scale_offsets, int64_t n_out1, int64_t k1, int64_t n_out2,
                             int64_t k2, int64_t tile_m, void* workspace,
                             size_t workspace_bytes, i8moe_stream_t stream) {
  I8_REQUIRE(tile_m > 0, "route_for_gemm: tile_m must be positive");
  I8_REQUIRE(expert_offsets && problem_sizes13 && problem_sizes2 && scale_offsets,
             "route_for_gemm: every output must be given");
  return launch_route_fused(topk_ids, token_expert_indices, expert_map, n_token, topk, n_expert,
                            n_local_expert, expert_first_token_offset, inv_permuted_idx,
                            permuted_idx, workspace, workspace_bytes,
                            static_cast<cudaStream_t>(stream), expert_offsets, problem_sizes13,
                            problem_sizes2, scale_offsets, static_cast<int>(n_out1),
                            static_cast<int>(k1), static_cast<int>(n_out2), static_cast<int>(k2),
                            static_cast<int>(tile_m));
}

int i8moe_moe_permute(const void* input, int dtype, int64_t n_hidden, const int32_t* topk_ids,
                      const int32_t* token_expert_indices, const int32_t* expert_map,
                      int64_t n_token, int64_t topk, int64_t n_expert, int64_t n_local_expert,
                      void* permuted_input, int64_t* expert_first_token_offset,
                      int32_t* inv_permuted_idx, int32_t* permuted_idx, void* workspace,
                      size_t workspace_bytes, i8moe_stream_t stream) {
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16 || dtype == I8MOE_FP32,
               "moe_permute: unsupported dtype");
  const int64_t row_bytes = n_hidden * dtype_size(dtype);
  I8_REQUIRE(row_bytes % 16 == 0, "moe_permute: hidden row must be a multiple of 16 bytes");
  I8_REQUIRE((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(permuted_input)) %
                     16 == 0,
                 "moe_permute: input/output must be 16-byte aligned");
  int rc = launch_route(topk_ids, token_expert_indices, expert_map, n_token, topk, n_expert,
                        n_local_expert, expert_first_token_offset, inv_permuted_idx,
                        permuted_idx, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream), FusedExtras{});
  if (rc != I8MOE_OK) return rc;
  const int64_t R = n_token * topk;
  if (R == 0 || n_hidden == 0) return I8MOE_OK;
  const int vpr = static_cast<int>(row_bytes / 16);
  const int threads = std::min(256, std::max(32, vpr));
  const int grid = static_cast<int>(std::min<int64_t>(R, 148 * 16));
  expand_rows<16><<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(input), static_cast<uint4*>(permuted_input), permuted_idx,
      expert_first_token_offset, static_cast<int>(n_local_expert), static_cast<int>(R),
      static_cast<int>(topk), vpr, expert_map != nullptr ? 1 : 0);
  return check_launch("expand_rows");
}

int i8moe_moe_unpermute(const void* permuted_hidden, int dtype, const float* topk_weights,
                        const int32_t* inv_permuted_idx,
                        const int64_t* expert_first_token_offset, int64_t n_local_expert,
                        int64_t n_token, int64_t topk, int64_t n_hidden, void* out,
                        i8moe_stream_t stream) {
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16 || dtype == I8MOE_FP32,
               "moe_unpermute: unsupported dtype");
  I8_REQUIRE(topk >= 1, "moe_unpermute: topk must be positive");
  I8_REQUIRE(n_token >= 0 && n_token < (int64_t(1) << 31), "moe_unpermute: bad n_token");
  const int64_t row_bytes = n_hidden * dtype_size(dtype);
  I8_REQUIRE(row_bytes % 16 == 0, "moe_unpermute: hidden row must be a multiple of 16 bytes");
  I8_REQUIRE((reinterpret_cast<uintptr_t>(permuted_hidden) | reinterpret_cast<uintptr_t>(out)) %
                     16 == 0,
                 "moe_unpermute: tensors must be 16-byte aligned");
  if (n_token == 0 || n_hidden == 0) return I8MOE_OK;
  const int vpr = static_cast<int>(row_bytes / 16);
  const int threads = std::min(256, std::max(32, ((vpr + 31) / 32) * 32));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nl = static_cast<int>(n_local_expert);
  const int k = static_cast<int>(topk);
  const dim3 grid(static_cast<unsigned>((n_token + 1) / 2));
  if (dtype == I8MOE_BF16) {
    unpermute_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(permuted_hidden), topk_weights, inv_permuted_idx,
        expert_first_token_offset, nl, k, vpr, static_cast<__nv_bfloat16*>(out), static_cast<int>(n_token));
  } else if (dtype == I8MOE_FP16) {
    unpermute_kernel<__half><<<grid, threads, 0, st>>>(
        static_cast<const __half*>(permuted_hidden), topk_weights, inv_permuted_idx,
        expert_first_token_offset, nl, k, vpr, static_cast<__half*>(out), static_cast<int>(n_token));
  } else {
    unpermute_kernel<float><<<grid, threads, 0, st>>>(
        static_cast<const float*>(permuted_hidden), topk_weights, inv_permuted_idx,
        expert_first_token_offset, nl, k, vpr, static_cast<float*>(out), static_cast<int>(n_token));
  }
  return check_launch("moe_unpermute");
}

int i8moe_silu_and_mul(void* out, const void* input, int dtype, int64_t n_rows, int64_t d,
                       i8moe_stream_t stream) {
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16 || dtype == I8MOE_FP32,
               "silu_and_mul: unsupported dtype");
  I8_REQUIRE((d * dtype_size(dtype)) % 16 == 0,
             "silu_and_mul: d must be a multiple of 16 bytes of elements");
  I8_REQUIRE((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(input)) % 16 == 0,
             "silu_and_mul: tensors must be 16-byte aligned");
  if (n_rows == 0 || d == 0) return I8MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t vecs = n_rows * d * dtype_size(dtype) / 16;
  const int grid = static_cast<int>(std::min<int64_t>((vecs + 255) / 256, 148 * 16));
  if (dtype == I8MOE_BF16) {
    silu_mul_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(input), static_cast<__nv_bfloat16*>(out), n_rows,
        static_cast<int>(d));
  } else if (dtype == I8MOE_FP16) {
    silu_mul_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(input),
                                                  static_cast<__half*>(out), n_rows,
                                                  static_cast<int>(d));
  } else {
    silu_mul_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(input),
                                                 static_cast<float*>(out), n_rows,
                                                 static_cast<int>(d));
  }
  return check_launch("silu_and_mul");
}

}  // extern "C"
