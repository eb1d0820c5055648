// umma_issue.cu -- how fast one CTA can issue tcgen05.mma (kind::f16, M = 128, K = 16,
// bf16 operands from zeroed 128-byte-swizzled shared memory, fp32 accumulators in
// tensor memory).  One thread issues 24 MMAs; clock64 stamps give the issue cost
// per instruction, how far issue runs ahead of execution (queue depth) and the
// completion time.  Mode 0 stamps every issue, mode 1 only start and end, mode 2
// has two warps issue at once into separate accumulators.  Uses the kernel's own
// PTX wrappers (csrc/sm100_ptx.cuh).  Every wait is bounded.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -Iampere_flash_attention_from_scratch_b200/csrc -o umma_issue \
//        ampere_flash_attention_from_scratch_b200/microbench/umma_issue.cu && ./umma_issue
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "sm100_ptx.cuh"

using namespace afa100;

constexpr int NMMA = 24;

template <int N, int MODE>
__global__ void __launch_bounds__(128, 1) bench(unsigned long long* out, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  for (int i = threadIdx.x; i < 49152 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(smem)[i] = 0u;
  const uint32_t bar0 = sbase + 49152;
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 49152 + 64);
  if (threadIdx.x == 0) { mbar_init(bar0, 1); mbar_init(bar0 + 8, 1); fence_mbarrier_init(); }
  if (threadIdx.x < 32) { tmem_alloc(smem_u32(slot), 512); tmem_relinquish(); }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(slot);
  const int warp = threadIdx.x / 32;
  const bool active = MODE == 2 ? warp < 2 : warp == 0;
  if (active) {
    const uint32_t leader = (threadIdx.x & 31) == 0 ? 1u : 0u;
    constexpr uint32_t idesc = idesc_f16_f32(128, N, true, false);
    const uint32_t d = tmem + (warp == 1 ? 256u : 0u);
    const uint32_t bar = bar0 + 8u * warp;
    unsigned long long t[NMMA + 1];
    t[0] = clock64();
#pragma unroll
    for (int i = 0; i < NMMA; ++i) {
      const uint32_t off = (i % 4) * 32u;
      umma_f16_ss(d, sdesc_lo(sbase + off, 16), sdesc_lo(sbase + 16384 + off, 16), idesc, i > 0 ? 1u : 0u, leader);
      if (MODE == 0) t[i + 1] = clock64();
    }
    const unsigned long long ti = clock64();
    umma_commit(bar, leader);
    bool done = false;
    for (int k = 0; k < (1 << 22) && !done; ++k) done = mbar_try_wait(bar, 0);
    const unsigned long long te = clock64();
    if (!done && leader) *status = 1;
    if (leader) {
      unsigned long long* o = out + warp * 64;
      if (MODE == 0) for (int i = 0; i <= NMMA; ++i) o[i] = t[i] - t[0];
      o[NMMA + 1] = ti - t[0];
      o[NMMA + 2] = te - t[0];
      o[NMMA + 3] = t[0];
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) { tc_fence_after_sync(); tmem_dealloc(tmem, 512); }
}

template <int N, int MODE>
void run(const char* name) {
  unsigned long long* d; int* st;
  cudaMalloc(&d, 128 * 8); cudaMalloc(&st, 4); cudaMemset(st, 0, 4); cudaMemset(d, 0, 128 * 8);
  const int smem = 49152 + 1024 + 1024;
  cudaFuncSetAttribute(bench<N, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  for (int rep = 0; rep < 3; ++rep) bench<N, MODE><<<1, 128, smem>>>(d, st);
  cudaError_t e = cudaDeviceSynchronize();
  unsigned long long h[128]; int hs = 0;
  cudaMemcpy(h, d, 128 * 8, cudaMemcpyDeviceToHost); cudaMemcpy(&hs, st, 4, cudaMemcpyDeviceToHost);
  printf("%s: %s status %d\n", name, cudaGetErrorString(e), hs);
  for (int w = 0; w < (MODE == 2 ? 2 : 1); ++w) {
    const unsigned long long* o = h + w * 64;
    long long skew = (long long)o[NMMA + 3] - (long long)h[NMMA + 3];
    printf("  warp %d (start %+lld): issue of %d MMAs done %llu cycles (%.1f per MMA), completion %llu", w, skew, NMMA,
           o[NMMA + 1], o[NMMA + 1] / double(NMMA), o[NMMA + 2]);
    if (MODE == 0) {
      printf("\n    deltas:");
      for (int i = 1; i <= NMMA; ++i) printf(" %llu", o[i] - o[i - 1]);
    }
    printf("\n");
  }
  cudaFree(d); cudaFree(st);
}

int main() {
  run<128, 0>("N128 one warp, stamps per issue");
  run<128, 1>("N128 one warp, no stamps");
  run<64, 1>("N64 one warp, no stamps");
  run<256, 1>("N256 one warp, no stamps");
  run<128, 2>("N128 two warps");
  run<64, 2>("N64 two warps");
  return 0;
}
