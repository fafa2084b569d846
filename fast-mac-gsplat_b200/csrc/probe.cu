// FP32 throughput probe: the measured denominator of the compositing kernels'
// FP32 roofline. Every thread runs kChains independent chains of fused
// multiply-adds (scalar fma.rn.f32, or packed fma.rn.f32x2 doing two per
// instruction) on a full-occupancy grid, so the FMA pipes, not latency, bound
// it. Written as bare PTX so the compiler keeps every operation. No reference
// counterpart.
#include "gsb_common.cuh"
#include "gsb_host.cuh"

namespace gsb {
namespace {

constexpr int kProbeThreads = 256;
constexpr int kChains = 8;

template <bool kPacked>
__global__ void __launch_bounds__(kProbeThreads) k_fma_probe(float* __restrict__ out, int iters, float seed) {
  const float m = 0.999999f, c = 1e-7f;
  if (kPacked) {
    unsigned long long v[kChains], mm, cc;
    asm("mov.b64 %0, {%1, %1};" : "=l"(mm) : "f"(m));
    asm("mov.b64 %0, {%1, %1};" : "=l"(cc) : "f"(c));
#pragma unroll
    for (int k = 0; k < kChains; ++k) {
      const float x = seed + (float)(threadIdx.x * kChains + k);
      asm("mov.b64 %0, {%1, %2};" : "=l"(v[k]) : "f"(x), "f"(x + 0.5f));
    }
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int k = 0; k < kChains; ++k) asm volatile("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(v[k]) : "l"(mm), "l"(cc));
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < kChains; ++k) {
      float lo, hi;
      asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v[k]));
      s += lo + hi;
    }
    out[blockIdx.x * kProbeThreads + threadIdx.x] = s;
  } else {
    float v[kChains];
#pragma unroll
    for (int k = 0; k < kChains; ++k) v[k] = seed + (float)(threadIdx.x * kChains + k);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int k = 0; k < kChains; ++k) asm volatile("fma.rn.f32 %0, %0, %1, %2;" : "+f"(v[k]) : "f"(m), "f"(c));
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < kChains; ++k) s += v[k];
    out[blockIdx.x * kProbeThreads + threadIdx.x] = s;
  }
}

}  // namespace
}  // namespace gsb

// Grid of the probe: blocks_per_sm x SMs blocks of 256 threads; `out` holds one
// float per thread (gsb_fma_probe_out_floats). FLOPs per launch =
// blocks x 256 x iters x 8 chains x 2 (x 2 more when packed).
extern "C" int64_t gsb_fma_probe_out_floats(int32_t blocks_per_sm) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int64_t)sms * blocks_per_sm * gsb::kProbeThreads;
}

extern "C" int gsb_fma_probe(int32_t packed, int32_t blocks_per_sm, int32_t iters, float* out, void* stream) {
  if (out == nullptr || blocks_per_sm < 1 || blocks_per_sm > 64 || iters < 1) return GSB_ERR_INVALID_ARGUMENT;
  const int64_t threads = gsb_fma_probe_out_floats(blocks_per_sm);
  const int grid = (int)(threads / gsb::kProbeThreads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (packed)
    gsb::k_fma_probe<true><<<grid, gsb::kProbeThreads, 0, s>>>(out, iters, 1.0f);
  else
    gsb::k_fma_probe<false><<<grid, gsb::kProbeThreads, 0, s>>>(out, iters, 1.0f);
  gsb::note_launches(1);
  return gsb::cuda_status(cudaGetLastError());
}
