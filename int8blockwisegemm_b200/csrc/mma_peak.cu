// Dense INT8 tensor-core peak of this device, measured: tcgen05.mma
// kind::i8 issued back to back from operands resident in shared memory, no
// operand loads, no epilogue.  One persistent CTA per SM (or one CTA pair per
// two SMs with cta_group::2, M = 256); each CTA issues `steps` x four
// M x 256 x 32 MMAs into one TMEM accumulator and waits for their completion
// (bounded).  The host times the launch: ops = 2 * 128 * 256 * 128 * steps
// per CTA.  This is the denominator of the INT8 roofline fractions that
// bench.py reports; the GEMM kernels' own operand stream and epilogue are
// what they add on top of it.
#include "common.cuh"

namespace i8moe {

static __device__ unsigned g_err_peak;

namespace {

constexpr int kPeakThreads = 128;
constexpr int kPeakN = 256;
constexpr int kPeakSmem = 128 * 128 + kPeakN * 128 + 1024;  // A, B int8 + alignment

template <int CG>
__global__ void __launch_bounds__(kPeakThreads, 1) mma_peak_kernel(int64_t steps) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  // operands: zeros (the values do not change the MMA rate)
  for (int i = threadIdx.x; i < (128 * 128 + kPeakN / CG * 128) / 16; i += kPeakThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    mbar_fence_init();
  }
  fence_proxy_async_smem();  // generic-proxy zeros visible to the tensor core
  if constexpr (CG == 2) cluster_sync();
  __syncthreads();
  if (warp == 0) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(smem_u32(&tmem_slot), kPeakN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(&tmem_slot), kPeakN);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t a = smem_u32(smem);
  const uint32_t b = a + 128 * 128;
  const bool leader = CG == 1 || cluster_ctarank() == 0;
  if (threadIdx.x == 0 && leader) {
    constexpr uint32_t idesc = idesc_i8(128 * CG, kPeakN);
    for (int64_t s = 0; s < steps; ++s) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t ad = sw128_kmajor_desc(a + 32 * k);
        const uint64_t bd = sw128_kmajor_desc(b + 32 * k);
        if constexpr (CG == 2)
          umma_i8_pair(tmem, ad, bd, idesc, (s > 0 || k > 0) ? 1u : 0u);
        else
          umma_i8(tmem, ad, bd, idesc, (s > 0 || k > 0) ? 1u : 0u);
      }
    }
    if constexpr (CG == 2) {
      umma_commit_pair(mapa_shared(smem_u32(&bar), 0));
      umma_commit_pair(mapa_shared(smem_u32(&bar), 1));
    } else {
      umma_commit(smem_u32(&bar));
    }
  }
  if (threadIdx.x == 0) {
    // both CTAs of a pair wait for the leader's MMAs (they read both CTAs'
    // shared memory and write both CTAs' TMEM)
    mbar_wait(smem_u32(&bar), 0, reinterpret_cast<volatile int*>(&abort_flag), &g_err_peak,
              kErrMmaTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem, kPeakN);
    else
      tmem_dealloc(tmem, kPeakN);
  }
}

}  // namespace

int read_peak_error(uint32_t* w, int clear) {
  unsigned v = 0;
  I8_CUDA(cudaMemcpyFromSymbol(&v, g_err_peak, sizeof(v)));
  if (clear) {
    unsigned z = 0;
    I8_CUDA(cudaMemcpyToSymbol(g_err_peak, &z, sizeof(z)));
  }
  *w = v;
  return I8MOE_OK;
}

}  // namespace i8moe

using namespace i8moe;

extern "C" {

int i8moe_int8_mma_peak(int64_t steps, int cta_group, int64_t* n_cta, i8moe_stream_t stream) {
  I8_REQUIRE(steps >= 1 && steps <= (int64_t(1) << 30), "mma peak: steps must be in [1, 2^30]");
  I8_REQUIRE(cta_group == 1 || cta_group == 2, "mma peak: cta_group must be 1 or 2");
  const int dev = current_device();
  int major = 0;
  I8_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  I8_REQUIRE(major == 10, "mma peak: needs an sm_100 device");
  const int sms = num_sms(dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cta_group == 1) {
    auto k = mma_peak_kernel<1>;
    I8_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem));
    k<<<sms, kPeakThreads, kPeakSmem, st>>>(steps);
    if (n_cta) *n_cta = sms;
  } else {
    auto k = mma_peak_kernel<2>;
    I8_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * static_cast<unsigned>(sms / 2));
    cfg.blockDim = dim3(kPeakThreads);
    cfg.dynamicSmemBytes = kPeakSmem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    I8_CUDA(cudaLaunchKernelEx(&cfg, k, steps));
    if (n_cta) *n_cta = 2 * (sms / 2);
  }
  return check_launch("mma_peak_kernel");
}

}  // extern "C"
