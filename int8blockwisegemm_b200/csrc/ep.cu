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
#include <algorithm>

#include "common.cuh"

namespace i8moe {
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
