// Expert-parallel token exchange: the device-side bookkeeping around the
// NCCL all-to-alls of the dispatch and the combine.
//
//   ep_plan     one CTA per destination rank d: token t goes to d when one of
//               its top-k experts lies in [d*n_local, (d+1)*n_local).  A
//               block-wide scan over the tokens gives every member its slot
//               in d's send segment (token order) -- pos[t, d], or -1 -- the
//               segment's token list and its length.
//   ep_pack     gathers the rows (and their top-k ids and weights) of every
//               segment into one contiguous send buffer, segment by segment.
//   ep_combine  out[t] = dtype(sum over ranks d, in rank order, of the
//               partial row that came back from d), fp32 accumulation.
//
// These replace host-driven torch glue (nonzero, index_select, index_add_)
// and keep the exchange to a single host synchronisation: the segment
// lengths that size the NCCL transfers.
//
// The peer-memory exchange (ep_p2p_*) needs no NCCL call and no host
// synchronisation at all.  Every rank owns one device region, mapped into
// every other rank's process through CUDA IPC (plain NVLink peer access):
//
//   rows   [C, K]     receive rows         (written by the sources)
//   ids    [C, k]     their top-k ids       (written by the sources)
//   w      [C, k]     their top-k weights   (written by the sources)
//   out    [2][C, K]  local forward output, by step parity (read by sources;
//                     the partial-row combine)
//   mm2    [2][C*k, K], inv [2][C, k]
//                     the w2 GEMM output and the routing's inverse map, by
//                     step parity (read by sources; the top-k combine)
//   inbox  [2][P][P]  every source's segment lengths, by step parity
//   flags  [3][P]     epochs: lengths posted, rows posted, output ready
//   epoch, counter    this rank's step number and a CTA completion counter
//
// with C = P x (tokens per rank) rows of capacity.  A step is
//   dispatch: post the P lengths to every peer, wait (bounded) for all of
//             theirs, then store every row straight into its destination's
//             receive buffer at its final offset (sources in rank order,
//             tokens in order: the same row order as the NCCL path); the
//             last CTA to finish raises this rank's "rows posted" flag at
//             every peer;
//   wait:     until every source has posted its rows; rows past the
//             received ones get a non-local expert id (the local routing
//             skips them);
//   (the unchanged single-GPU forward over the C receive rows)
//   ready:    raise this rank's "output ready" flag at every peer;
//   combine:  wait for every destination's output, then sum this rank's
//             tokens' partial rows, read from the peers' memory, in rank
//             order in fp32 -- or, with the top-k combine, the local forward
//             stops after the w2 GEMM and the combine is the whole top-k
//             weighted unpermute over the peers' mm2 rows, so the output
//             equals a single-GPU forward bit for bit.
// Flags carry the step number and waits test flag >= step, so a peer that
// runs a step ahead never blocks one behind; a peer can never run two
// steps ahead (a step's dispatch needs every peer's previous output to
// have been combined).  Every wait gives up after kP2PTimeoutNs with an
// error bit (i8moe_device_error) instead of hanging.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace i8moe {

static __device__ unsigned g_err_ep;

int read_ep_error(uint32_t* w, int clear) {
  unsigned v = 0;
  I8_CUDA(cudaMemcpyFromSymbol(&v, g_err_ep, sizeof(v)));
  if (clear) {
    unsigned z = 0;
    I8_CUDA(cudaMemcpyToSymbol(g_err_ep, &z, sizeof(z)));
  }
  *w = v;
  return I8MOE_OK;
}

namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxRanks = 32;

struct RankOffsets {
  int64_t off[kMaxRanks + 1];  // segment starts in the packed send / returned buffer
};

__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int32_t* __restrict__ ids,
                                                               int T, int k, int n_local, int P,
                                                               int32_t* __restrict__ pos,
                                                               int32_t* __restrict__ list,
                                                               int32_t* __restrict__ counts) {
  __shared__ int s_warp[kPlanThreads / 32];
  __shared__ int s_base;
  const int d = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += kPlanThreads) {
    const int t = t0 + tid;
    int member = 0;
    if (t < T) {
      for (int j = 0; j < k; ++j) {
        const int e = __ldg(ids + static_cast<int64_t>(t) * k + j);
        member |= (e >= 0 && e / n_local == d) ? 1 : 0;
      }
    }
    // block-wide exclusive scan of `member`
    const unsigned bal = __ballot_sync(0xffffffffu, member);
    const int in_warp = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) s_warp[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
      int v = s_warp[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      s_warp[lane] = v;  // inclusive
    }
    __syncthreads();
    const int base = s_base;
    const int before = (warp > 0 ? s_warp[warp - 1] : 0) + in_warp;
    if (t < T) {
      const int p = member ? base + before : -1;
      pos[static_cast<int64_t>(t) * P + d] = p;
      if (member) list[static_cast<int64_t>(d) * T + p] = t;
    }
    __syncthreads();
    if (tid == 0) s_base = base + s_warp[kPlanThreads / 32 - 1];
    __syncthreads();
  }
  if (tid == 0) counts[d] = s_base;
}

// One warp per packed row: the 16-byte chunks of the row, then one meta row
// of its k ids followed by the bits of its k weights.
__global__ void __launch_bounds__(256) ep_pack_kernel(
    const uint4* __restrict__ hidden, int64_t row_chunks, const int32_t* __restrict__ ids,
    const float* __restrict__ weights, int k, const int32_t* __restrict__ list, int T, int P,
    RankOffsets ro, uint4* __restrict__ send_rows, int32_t* __restrict__ send_meta) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= ro.off[P]) return;
  int d = 0;
  while (d + 1 < P && ro.off[d + 1] <= row) ++d;
  const int t = __ldg(list + static_cast<int64_t>(d) * T + (row - ro.off[d]));
  const uint4* src = hidden + static_cast<int64_t>(t) * row_chunks;
  uint4* dst = send_rows + row * row_chunks;
  for (int64_t c = lane; c < row_chunks; c += 32) dst[c] = __ldg(src + c);
  if (lane < k) {
    send_meta[row * 2 * k + lane] = __ldg(ids + static_cast<int64_t>(t) * k + lane);
    send_meta[row * 2 * k + k + lane] =
        __float_as_int(__ldg(weights + static_cast<int64_t>(t) * k + lane));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ep_combine_kernel(const T* __restrict__ back,
                                                         const int32_t* __restrict__ pos,
                                                         int n_token, int P, int K, RankOffsets ro,
                                                         T* __restrict__ out) {
  constexpr int EPC = 8;  // 16-bit elements per 16-byte chunk
  const int t = blockIdx.x;
  if (t >= n_token) return;
  int64_t rows[kMaxRanks];
  int nr = 0;
  for (int d = 0; d < P; ++d) {
    const int p = __ldg(pos + static_cast<int64_t>(t) * P + d);
    if (p >= 0) rows[nr++] = ro.off[d] + p;
  }
  for (int c = threadIdx.x; c * EPC < K; c += blockDim.x) {
    float acc[EPC];
#pragma unroll
    for (int i = 0; i < EPC; ++i) acc[i] = 0.f;
    for (int r = 0; r < nr; ++r) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(back + rows[r] * K) + c);
      const T* x = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int i = 0; i < EPC; ++i) acc[i] += Num<T>::to_f(x[i]);
    }
    uint4 o;
    T* y = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int i = 0; i < EPC; ++i) y[i] = Num<T>::from_f(acc[i]);
    reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * K)[c] = o;
  }
}

// ---------------------------------------------------------------------------
// peer-memory exchange
// ---------------------------------------------------------------------------
constexpr uint64_t kP2PTimeoutNs = 2000000000ull;  // 2 s
constexpr unsigned kErrPeerTimeout = 1u << 6;

struct P2PArgs {
  uint8_t* base[kMaxRanks];  // every rank's region as mapped in this process
  int P, rank;
  int T;                     // tokens of this rank
  int C;                     // receive capacity (rows)
  int k, K, esize;           // top-k, hidden, bytes per hidden element
  int pad_id;                // a global expert id no local expert has
  int par;                   // step parity
  int64_t off_rows, off_ids, off_w, off_out, out_bytes, off_inbox, off_flags, off_epoch;
  int64_t off_mm2, mm2_bytes, off_inv, inv_bytes;  // top-k combine (per parity)
};

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t* flag_ptr(const P2PArgs& a, int owner, int kind, int src) {
  return reinterpret_cast<uint64_t*>(a.base[owner] + a.off_flags) + kind * a.P + src;
}
__device__ __forceinline__ int32_t* inbox_ptr(const P2PArgs& a, int owner) {
  return reinterpret_cast<int32_t*>(a.base[owner] + a.off_inbox) + a.par * a.P * a.P;
}
__device__ __forceinline__ uint64_t my_epoch(const P2PArgs& a) {
  return *reinterpret_cast<volatile uint64_t*>(a.base[a.rank] + a.off_epoch);
}
// one thread: until this rank's flags `kind` from every rank reach `ep`
__device__ bool wait_flags(const P2PArgs& a, int kind, uint64_t ep) {
  const uint64_t t0 = globaltimer();
  for (int s = 0; s < a.P; ++s) {
    const uint64_t* f = flag_ptr(a, a.rank, kind, s);
    while (ld_acquire_sys(f) < ep) {
      if (globaltimer() - t0 > kP2PTimeoutNs) {
        atomicOr(&g_err_ep, kErrPeerTimeout);
        return false;
      }
    }
  }
  return true;
}
enum { kFlagCounts = 0, kFlagRows = 1, kFlagOut = 2 };

__global__ void ep_p2p_begin(const __grid_constant__ P2PArgs a) {
  uint64_t* e = reinterpret_cast<uint64_t*>(a.base[a.rank] + a.off_epoch);
  *e = *e + 1;
}

// Offsets of this rank's segment in every destination's receive buffer:
// off_to[d] = sum over sources s < rank of count[s][d] (shared memory).
__device__ void p2p_offsets(const P2PArgs& a, int* off_to) {
  const int32_t* inbox = inbox_ptr(a, a.rank);
  if (threadIdx.x < a.P) {
    const int d = threadIdx.x;
    int o = 0;
    for (int s = 0; s < a.rank; ++s) o += __ldcg(inbox + s * a.P + d);  // written by peers
    off_to[d] = o;
  }
}

__global__ void __launch_bounds__(256) ep_p2p_dispatch_kernel(const __grid_constant__ P2PArgs a, const uint4* __restrict__ hidden,
                                                              const int32_t* __restrict__ ids,
                                                              const float* __restrict__ w,
                                                              const int32_t* __restrict__ list,
                                                              const int32_t* __restrict__ counts,
                                                              unsigned* __restrict__ done_ctr) {
  __shared__ int s_off[kMaxRanks], s_seg[kMaxRanks + 1];
  __shared__ int s_ok;
  const uint64_t ep = my_epoch(a);
  if (blockIdx.x == 0 && threadIdx.x < a.P) {
    // post this rank's segment lengths to destination d, then the flag
    const int d = threadIdx.x;
    int32_t* dst = inbox_ptr(a, d) + a.rank * a.P;
    for (int j = 0; j < a.P; ++j) dst[j] = __ldg(counts + j);
    __threadfence_system();
    st_release_sys(flag_ptr(a, d, kFlagCounts, a.rank), ep);
  }
  if (threadIdx.x == 0) s_ok = wait_flags(a, kFlagCounts, ep) ? 1 : 0;
  __syncthreads();
  // A CTA whose wait gave up (the error word now says so) copies no rows but
  // still counts itself below: the persistent completion counter must see
  // every CTA of every launch, or a later step's "rows posted" flag would be
  // raised before all of that step's rows are stored.
  if (s_ok) p2p_offsets(a, s_off);
  if (threadIdx.x == 0) {
    int o = 0;
    for (int d = 0; d < a.P; ++d) {
      s_seg[d] = o;
      o += __ldg(counts + d);
    }
    s_seg[a.P] = s_ok ? o : 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t chunks = static_cast<int64_t>(a.K) * a.esize / 16;
  const int64_t n_rows = s_seg[a.P];
  const int wpb = blockDim.x / 32;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); g < n_rows;
       g += static_cast<int64_t>(gridDim.x) * wpb) {
    int d = 0;
    while (d + 1 < a.P && s_seg[d + 1] <= g) ++d;
    const int p = static_cast<int>(g - s_seg[d]);
    const int t = __ldg(list + static_cast<int64_t>(d) * a.T + p);
    const int64_t row = s_off[d] + p;  // in d's receive buffer
    if (row >= a.C) {  // capacity is P x tokens per rank, so never
      if (lane == 0) atomicOr(&g_err_ep, kErrBadIndex);
      continue;
    }
    const uint4* src = hidden + static_cast<int64_t>(t) * chunks;
    uint4* dst = reinterpret_cast<uint4*>(a.base[d] + a.off_rows) + row * chunks;
    // all of a lane's loads of the row go out before its peer stores
    constexpr int kU = 8;
    for (int64_t c0 = 0; c0 < chunks; c0 += 32 * kU) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < chunks) v[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < chunks) dst[c] = v[u];
      }
    }
    if (lane < a.k) {
      reinterpret_cast<int32_t*>(a.base[d] + a.off_ids)[row * a.k + lane] =
          __ldg(ids + static_cast<int64_t>(t) * a.k + lane);
      reinterpret_cast<float*>(a.base[d] + a.off_w)[row * a.k + lane] =
          __ldg(w + static_cast<int64_t>(t) * a.k + lane);
    }
  }
  // the last CTA to finish raises the "rows posted" flag at every peer
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned old = atomicAdd(done_ctr, 1u);
    if (old == gridDim.x - 1) {
      *done_ctr = 0u;
      __threadfence_system();
      for (int d = 0; d < a.P; ++d) st_release_sys(flag_ptr(a, d, kFlagRows, a.rank), ep);
    }
  }
}

// Until every source has posted its rows; then the receive rows past the
// received ones get a non-local expert id and weight 0.
__global__ void __launch_bounds__(256) ep_p2p_wait_kernel(const __grid_constant__ P2PArgs a) {
  __shared__ int s_ok;
  const uint64_t ep = my_epoch(a);
  if (threadIdx.x == 0) s_ok = wait_flags(a, kFlagRows, ep) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const int32_t* inbox = inbox_ptr(a, a.rank);
  int n_recv = 0;
  for (int s = 0; s < a.P; ++s) n_recv += __ldcg(inbox + s * a.P + a.rank);
  n_recv = min(n_recv, a.C);
  int32_t* rid = reinterpret_cast<int32_t*>(a.base[a.rank] + a.off_ids);
  float* rw = reinterpret_cast<float*>(a.base[a.rank] + a.off_w);
  const int64_t n_pad = static_cast<int64_t>(a.C - n_recv) * a.k;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_pad;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    rid[static_cast<int64_t>(n_recv) * a.k + i] = a.pad_id;
    rw[static_cast<int64_t>(n_recv) * a.k + i] = 0.0f;
  }
}

// This rank's local forward output (a previous kernel on the stream) is
// complete: raise the "output ready" flag at every peer.
__global__ void ep_p2p_ready_kernel(const __grid_constant__ P2PArgs a) {
  const uint64_t ep = my_epoch(a);
  __threadfence_system();
  if (threadIdx.x < a.P) st_release_sys(flag_ptr(a, threadIdx.x, kFlagOut, a.rank), ep);
}

// out[t] = dtype(sum over destinations d in rank order of d's output row
// off_to[d] + pos[t, d]), fp32 accumulation, rows read from peer memory.
template <typename T>
__global__ void __launch_bounds__(256) ep_p2p_combine_kernel(const __grid_constant__ P2PArgs a, const int32_t* __restrict__ pos,
                                                             T* __restrict__ out) {
  constexpr int EPC = 8;
  __shared__ int s_off[kMaxRanks];
  __shared__ int64_t s_row[kMaxRanks];  // this token's row in destination d's output, or -1
  __shared__ int s_ok;
  const uint64_t ep = my_epoch(a);
  if (threadIdx.x == 0) s_ok = wait_flags(a, kFlagOut, ep) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  p2p_offsets(a, s_off);
  __syncthreads();
  const int chunks = a.K / EPC;
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    if (threadIdx.x < a.P) {
      const int d = threadIdx.x;
      const int p = __ldg(pos + static_cast<int64_t>(t) * a.P + d);
      s_row[d] = (p >= 0 && s_off[d] + p < a.C) ? static_cast<int64_t>(s_off[d] + p) : -1;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      float acc[EPC];
#pragma unroll
      for (int i = 0; i < EPC; ++i) acc[i] = 0.f;
      // up to eight destinations' loads in flight together, then summed in rank order
      constexpr int kU = 8;
      for (int d0 = 0; d0 < a.P; d0 += kU) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int d = d0 + u;
          if (d < a.P && s_row[d] >= 0) {
            const T* src = reinterpret_cast<const T*>(a.base[d] + a.off_out + a.par * a.out_bytes) +
                           s_row[d] * a.K;
            v[u] = __ldcg(reinterpret_cast<const uint4*>(src) + c);  // peer memory, via L2
          }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int d = d0 + u;
          if (d < a.P && s_row[d] >= 0) {
            const T* x = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
            for (int i = 0; i < EPC; ++i) acc[i] += Num<T>::to_f(x[i]);
          }
        }
      }
      uint4 o;
      T* y = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int i = 0; i < EPC; ++i) y[i] = Num<T>::from_f(acc[i]);
      reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * a.K)[c] = o;
    }
    __syncthreads();  // s_row is rewritten for the next token
  }
}

// Top-k combine: the unpermute of every token of this rank, over the mm2
// rows of all ranks.  Slot j of token t was computed by rank
// d = ids[t, j] / n_local; the token is receive row off_to[d] + pos[t, d]
// there, and that rank's routing put the slot's mm2 row at
// inv_d[row * k + j].  out[t] = dtype(fma chain over j in top-k order of
// w[t, j] * mm2 row, from 0): the arithmetic of the single-GPU unpermute
// (moe_permute_unpermute_kernel.inl:133-190), so the output equals a
// single-GPU forward bit for bit.  mm2 rows are read from peer memory, up to
// eight slots in flight per thread.
template <typename T>
__global__ void __launch_bounds__(256) ep_p2p_combine_topk_kernel(
    const __grid_constant__ P2PArgs a, const int32_t* __restrict__ pos,
    const int32_t* __restrict__ ids, const float* __restrict__ w, int n_local,
    T* __restrict__ out) {
  constexpr int EPC = 8;
  constexpr int kMaxK = 32;
  __shared__ int s_off[kMaxRanks];
  __shared__ const uint4* s_src[kMaxK];  // slot j's mm2 row, or null (skipped)
  __shared__ float s_w[kMaxK];
  __shared__ int s_ok;
  const uint64_t ep = my_epoch(a);
  if (threadIdx.x == 0) s_ok = wait_flags(a, kFlagOut, ep) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  p2p_offsets(a, s_off);
  __syncthreads();
  const int chunks = a.K / EPC;
  const int64_t max_row = static_cast<int64_t>(a.C) * a.k;
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    if (threadIdx.x < a.k) {
      const int j = threadIdx.x;
      const int e = __ldg(ids + static_cast<int64_t>(t) * a.k + j);
      const int d = e >= 0 ? e / n_local : -1;
      const uint4* src = nullptr;
      if (d >= 0 && d < a.P) {
        const int p = __ldg(pos + static_cast<int64_t>(t) * a.P + d);
        const int64_t row = static_cast<int64_t>(s_off[d]) + p;
        if (p >= 0 && row < a.C) {
          const int32_t* inv =
              reinterpret_cast<const int32_t*>(a.base[d] + a.off_inv + a.par * a.inv_bytes);
          const int prow = __ldcg(inv + row * a.k + j);  // written by rank d
          if (prow >= 0 && prow < max_row)
            src = reinterpret_cast<const uint4*>(a.base[d] + a.off_mm2 + a.par * a.mm2_bytes) +
                  static_cast<int64_t>(prow) * chunks;
        }
      }
      if (src == nullptr) atomicOr(&g_err_ep, kErrBadIndex);  // every slot has an owner
      s_src[j] = src;
      s_w[j] = __ldg(w + static_cast<int64_t>(t) * a.k + j);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      float acc[EPC];
#pragma unroll
      for (int i = 0; i < EPC; ++i) acc[i] = 0.f;
      constexpr int kU = 8;
      for (int j0 = 0; j0 < a.k; j0 += kU) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int j = j0 + u;
          if (j < a.k && s_src[j] != nullptr) v[u] = __ldcg(s_src[j] + c);  // peer memory, via L2
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int j = j0 + u;
          if (j < a.k && s_src[j] != nullptr) {
            const float wt = s_w[j];
            const T* x = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
            for (int i = 0; i < EPC; ++i) acc[i] = fmaf(wt, Num<T>::to_f(x[i]), acc[i]);
          }
        }
      }
      uint4 o;
      T* y = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int i = 0; i < EPC; ++i) y[i] = Num<T>::from_f(acc[i]);
      reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * a.K)[c] = o;
    }
    __syncthreads();  // s_src / s_w are rewritten for the next token
  }
}

int offsets_from(const int64_t* counts, int P, RankOffsets* ro) {
  I8_REQUIRE(P >= 1 && P <= kMaxRanks, "ep: the group must have 1..%d ranks", kMaxRanks);
  ro->off[0] = 0;
  for (int d = 0; d < P; ++d) {
    I8_REQUIRE(counts[d] >= 0, "ep: negative segment length");
    ro->off[d + 1] = ro->off[d] + counts[d];
  }
  for (int d = P + 1; d <= kMaxRanks; ++d) ro->off[d] = ro->off[P];
  return I8MOE_OK;
}

}  // namespace
}  // namespace i8moe

using namespace i8moe;

extern "C" {

int i8moe_ep_plan(const int32_t* topk_ids, int64_t n_token, int64_t topk, int64_t n_local_expert,
                  int64_t n_rank, int32_t* pos, int32_t* token_list, int32_t* counts,
                  i8moe_stream_t stream) {
  I8_REQUIRE(n_rank >= 1 && n_rank <= kMaxRanks, "ep_plan: the group must have 1..%d ranks",
             kMaxRanks);
  I8_REQUIRE(n_token >= 0 && n_token < (int64_t(1) << 31) && topk >= 1 && n_local_expert >= 1,
             "ep_plan: bad arguments");
  ep_plan_kernel<<<static_cast<unsigned>(n_rank), kPlanThreads, 0,
                   static_cast<cudaStream_t>(stream)>>>(
      topk_ids, static_cast<int>(n_token), static_cast<int>(topk),
      static_cast<int>(n_local_expert), static_cast<int>(n_rank), pos, token_list, counts);
  return check_launch("ep_plan");
}

int i8moe_ep_pack(const void* hidden, int64_t row_bytes, const int32_t* topk_ids,
                  const float* topk_weights, int64_t topk, const int32_t* token_list,
                  int64_t n_token, int64_t n_rank, const int64_t* counts, void* send_rows,
                  int32_t* send_meta, i8moe_stream_t stream) {
  I8_REQUIRE(row_bytes > 0 && row_bytes % 16 == 0, "ep_pack: rows must be a multiple of 16 bytes");
  I8_REQUIRE((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(send_rows)) % 16 == 0,
             "ep_pack: row buffers must be 16-byte aligned");
  I8_REQUIRE(topk >= 1 && topk <= 32, "ep_pack: topk must be in [1, 32]");
  RankOffsets ro;
  int rc = offsets_from(counts, static_cast<int>(n_rank), &ro);  // host array
  if (rc) return rc;
  const int64_t rows = ro.off[n_rank];
  if (rows == 0) return I8MOE_OK;
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  ep_pack_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(hidden), row_bytes / 16, topk_ids, topk_weights,
      static_cast<int>(topk), token_list, static_cast<int>(n_token), static_cast<int>(n_rank), ro,
      static_cast<uint4*>(send_rows), send_meta);
  return check_launch("ep_pack");
}

int i8moe_ep_p2p_region_bytes(int64_t n_rank, int64_t capacity, int64_t topk, int64_t n_hidden,
                              int64_t elem_bytes, int combine, i8moe_ep_p2p_layout* layout) {
  I8_REQUIRE(n_rank >= 1 && n_rank <= kMaxRanks, "ep p2p: the group must have 1..%d ranks", kMaxRanks);
  I8_REQUIRE(capacity >= 1 && topk >= 1 && topk <= 32 && n_hidden >= 8 && elem_bytes == 2 &&
                 (n_hidden * elem_bytes) % 16 == 0,
             "ep p2p: bad shape");
  I8_REQUIRE(combine == I8MOE_EP_COMBINE_ROWS || combine == I8MOE_EP_COMBINE_TOPK,
             "ep p2p: combine must be I8MOE_EP_COMBINE_ROWS or I8MOE_EP_COMBINE_TOPK");
  I8_REQUIRE(capacity * topk < (int64_t(1) << 31), "ep p2p: capacity * topk must fit in int32");
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  const bool rows = combine == I8MOE_EP_COMBINE_ROWS;
  i8moe_ep_p2p_layout l{};
  int64_t o = 0;
  l.off_rows = o;  o = up(o + capacity * n_hidden * elem_bytes);
  l.off_ids = o;   o = up(o + capacity * topk * 4);
  l.off_w = o;     o = up(o + capacity * topk * 4);
  // partial rows (ROWS) or mm2 rows + inverse map (TOPK), one per parity
  l.off_out = o;   l.out_bytes = rows ? up(capacity * n_hidden * elem_bytes) : 0;
  o = up(o + 2 * l.out_bytes);
  l.off_mm2 = o;   l.mm2_bytes = rows ? 0 : up(capacity * topk * n_hidden * elem_bytes);
  o = up(o + 2 * l.mm2_bytes);
  l.off_inv = o;   l.inv_bytes = rows ? 0 : up(capacity * topk * 4);
  o = up(o + 2 * l.inv_bytes);
  l.off_inbox = o; o = up(o + 2 * n_rank * n_rank * 4);
  l.off_flags = o; o = up(o + 3 * n_rank * 8);
  l.off_epoch = o; o = up(o + 16);  // epoch (8 B), CTA completion counter (4 B)
  l.bytes = o;
  *layout = l;
  return I8MOE_OK;
}

int i8moe_ep_ipc_alloc(int64_t bytes, void** ptr, uint8_t* handle) {
  I8_REQUIRE(bytes > 0 && ptr != nullptr && handle != nullptr, "ep ipc: bad arguments");
  void* p = nullptr;
  I8_CUDA(cudaMalloc(&p, static_cast<size_t>(bytes)));
  cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(I8MOE_ERR_CUDA, std::string("ep ipc alloc: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == I8MOE_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return I8MOE_OK;
}

int i8moe_ep_ipc_open(const uint8_t* handle, void** ptr) {
  I8_REQUIRE(handle != nullptr && ptr != nullptr, "ep ipc: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  I8_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = p;
  return I8MOE_OK;
}

int i8moe_ep_ipc_close(void* ptr) {
  I8_CUDA(cudaIpcCloseMemHandle(ptr));
  return I8MOE_OK;
}

int i8moe_ep_ipc_free(void* ptr) {
  I8_CUDA(cudaFree(ptr));
  return I8MOE_OK;
}

}  // extern "C"

namespace {
int p2p_args(const i8moe_ep_p2p* x, int par, P2PArgs* a) {
  I8_REQUIRE(x != nullptr && x->n_rank >= 1 && x->n_rank <= kMaxRanks && x->rank >= 0 &&
                 x->rank < x->n_rank,
             "ep p2p: bad group");
  I8_REQUIRE(x->capacity >= 1 && x->topk >= 1 && x->topk <= 32 && x->elem_bytes == 2,
             "ep p2p: bad shape");
  *a = P2PArgs{};
  for (int d = 0; d < x->n_rank; ++d) {
    I8_REQUIRE(x->bases[d] != nullptr, "ep p2p: region of rank %d is not mapped", d);
    a->base[d] = static_cast<uint8_t*>(x->bases[d]);
  }
  a->P = static_cast<int>(x->n_rank);
  a->rank = static_cast<int>(x->rank);
  a->T = static_cast<int>(x->n_token);
  a->C = static_cast<int>(x->capacity);
  a->k = static_cast<int>(x->topk);
  a->K = static_cast<int>(x->n_hidden);
  a->esize = static_cast<int>(x->elem_bytes);
  a->pad_id = static_cast<int>(x->pad_expert);
  a->par = par & 1;
  a->off_rows = x->layout.off_rows;
  a->off_ids = x->layout.off_ids;
  a->off_w = x->layout.off_w;
  a->off_out = x->layout.off_out;
  a->out_bytes = x->layout.out_bytes;
  a->off_inbox = x->layout.off_inbox;
  a->off_flags = x->layout.off_flags;
  a->off_epoch = x->layout.off_epoch;
  a->off_mm2 = x->layout.off_mm2;
  a->mm2_bytes = x->layout.mm2_bytes;
  a->off_inv = x->layout.off_inv;
  a->inv_bytes = x->layout.inv_bytes;
  return I8MOE_OK;
}
}  // namespace

extern "C" {

int i8moe_ep_p2p_dispatch(const i8moe_ep_p2p* x, int par, const void* hidden,
                          const int32_t* topk_ids, const float* topk_weights,
                          const int32_t* token_list, const int32_t* counts,
                          i8moe_stream_t stream) {
  P2PArgs a;
  int rc = p2p_args(x, par, &a);
  if (rc) return rc;
  I8_REQUIRE(reinterpret_cast<uintptr_t>(hidden) % 16 == 0, "ep p2p: hidden must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ep_p2p_begin<<<1, 1, 0, st>>>(a);
  rc = check_launch("ep_p2p_begin");
  if (rc) return rc;
  unsigned* ctr = reinterpret_cast<unsigned*>(a.base[a.rank] + a.off_epoch + 8);
  const unsigned grid = static_cast<unsigned>(2 * num_sms(current_device()));
  ep_p2p_dispatch_kernel<<<grid, 256, 0, st>>>(a, static_cast<const uint4*>(hidden), topk_ids,
                                               topk_weights, token_list, counts, ctr);
  return check_launch("ep_p2p_dispatch");
}

int i8moe_ep_p2p_wait(const i8moe_ep_p2p* x, int par, i8moe_stream_t stream) {
  P2PArgs a;
  int rc = p2p_args(x, par, &a);
  if (rc) return rc;
  ep_p2p_wait_kernel<<<static_cast<unsigned>(num_sms(current_device())), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("ep_p2p_wait");
}

int i8moe_ep_p2p_ready(const i8moe_ep_p2p* x, int par, i8moe_stream_t stream) {
  P2PArgs a;
  int rc = p2p_args(x, par, &a);
  if (rc) return rc;
  ep_p2p_ready_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("ep_p2p_ready");
}

int i8moe_ep_p2p_combine(const i8moe_ep_p2p* x, int par, int dtype, const int32_t* pos, void* out,
                         i8moe_stream_t stream) {
  P2PArgs a;
  int rc = p2p_args(x, par, &a);
  if (rc) return rc;
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16, "ep p2p combine: bfloat16 or float16 rows");
  I8_REQUIRE(a.K % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0,
             "ep p2p combine: 16-byte rows");
  I8_REQUIRE(x->layout.out_bytes >= static_cast<int64_t>(a.C) * a.K * a.esize,
             "ep p2p combine: the region was not sized with I8MOE_EP_COMBINE_ROWS");
  if (a.T == 0) return I8MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(a.T, 4 * num_sms(current_device())));
  if (dtype == I8MOE_BF16)
    ep_p2p_combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a, pos, static_cast<__nv_bfloat16*>(out));
  else
    ep_p2p_combine_kernel<__half><<<grid, 256, 0, st>>>(a, pos, static_cast<__half*>(out));
  return check_launch("ep_p2p_combine");
}

int i8moe_ep_p2p_combine_topk(const i8moe_ep_p2p* x, int par, int dtype, const int32_t* pos,
                              const int32_t* topk_ids, const float* topk_weights,
                              int64_t n_local_expert, void* out, i8moe_stream_t stream) {
  P2PArgs a;
  int rc = p2p_args(x, par, &a);
  if (rc) return rc;
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16, "ep p2p combine: bfloat16 or float16 rows");
  I8_REQUIRE(a.K % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0,
             "ep p2p combine: 16-byte rows");
  I8_REQUIRE(x->layout.mm2_bytes >= static_cast<int64_t>(a.C) * a.k * a.K * a.esize &&
                 x->layout.inv_bytes >= static_cast<int64_t>(a.C) * a.k * 4,
             "ep p2p combine_topk: the region was not sized with I8MOE_EP_COMBINE_TOPK");
  I8_REQUIRE(n_local_expert >= 1 && n_local_expert < (int64_t(1) << 31),
             "ep p2p combine_topk: bad n_local_expert");
  if (a.T == 0) return I8MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(a.T, 4 * num_sms(current_device())));
  const int nl = static_cast<int>(n_local_expert);
  if (dtype == I8MOE_BF16)
    ep_p2p_combine_topk_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        a, pos, topk_ids, topk_weights, nl, static_cast<__nv_bfloat16*>(out));
  else
    ep_p2p_combine_topk_kernel<__half><<<grid, 256, 0, st>>>(a, pos, topk_ids, topk_weights, nl,
                                                             static_cast<__half*>(out));
  return check_launch("ep_p2p_combine_topk");
}

int i8moe_ep_combine(const void* back, int dtype, const int32_t* pos, int64_t n_token,
                     int64_t n_rank, const int64_t* counts, int64_t n_hidden, void* out,
                     i8moe_stream_t stream) {
  I8_REQUIRE(dtype == I8MOE_BF16 || dtype == I8MOE_FP16, "ep_combine: bfloat16 or float16 rows");
  I8_REQUIRE(n_hidden % 8 == 0, "ep_combine: n_hidden must be a multiple of 8");
  I8_REQUIRE((reinterpret_cast<uintptr_t>(back) | reinterpret_cast<uintptr_t>(out)) % 16 == 0,
             "ep_combine: buffers must be 16-byte aligned");
  RankOffsets ro;
  int rc = offsets_from(counts, static_cast<int>(n_rank), &ro);  // host array
  if (rc) return rc;
  if (n_token == 0) return I8MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(n_token);
  if (dtype == I8MOE_BF16)
    ep_combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(back), pos, static_cast<int>(n_token),
        static_cast<int>(n_rank), static_cast<int>(n_hidden), ro, static_cast<__nv_bfloat16*>(out));
  else
    ep_combine_kernel<__half><<<grid, 256, 0, st>>>(
        static_cast<const __half*>(back), pos, static_cast<int>(n_token),
        static_cast<int>(n_rank), static_cast<int>(n_hidden), ro, static_cast<__half*>(out));
  return check_launch("ep_combine");
}

}  // extern "C"
