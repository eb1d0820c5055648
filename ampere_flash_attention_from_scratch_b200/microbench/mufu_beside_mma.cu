// mufu_beside_mma.cu -- does the softmax arithmetic run as fast on an SM whose
// tensor core is busy?  One CTA per SM, 384 threads.  Warp 0 (when MMA is on)
// keeps tcgen05.mma (kind::f16, M = 128, N = 128, K = 16, bf16 operands from
// 128-byte-swizzled shared memory, fp32 accumulators in tensor memory) queued
// back to back (issue blocks while about four are queued), one commit at the end.
// Warps 4..4+4W-1 (W = 1 or 2 per SM sub-partition) run 2048 iterations of a
// 16-instruction arithmetic group (16 independent chains per thread) and
// stamp clock64 around it: `ex2.approx.ftz.f32` alone, the softmax's mix (16 ex2
// + 8 fma.rn.f32x2 + 8 cvt.rn.bf16x2.f32), or 16 fma.rn.f32x2.  Printed: cycles
// per 16-instruction group per sub-partition, averaged over the arithmetic warps
// of all SMs, and the cycles per MMA of warp 0's whole stream (also run alone,
// for SS N = 64 / 128 / 256, TS N = 128, one or two accumulators).  Every wait is
// bounded; a wait that runs out sets the status word.  Uses the kernel's own PTX
// wrappers (csrc/sm100_ptx.cuh).
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -Iampere_flash_attention_from_scratch_b200/csrc -o mufu_beside_mma \
//        ampere_flash_attention_from_scratch_b200/microbench/mufu_beside_mma.cu && ./mufu_beside_mma
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "sm100_ptx.cuh"

using namespace afa100;

constexpr int ITERS = 2048;
constexpr int kOperandBytes = 32768;  // A (16 KB) and B (16 KB) tiles
constexpr int kMmaGroups = 3200;      // 4 MMAs each: 12800 x 64 cycles, longer than any arithmetic loop

__device__ __forceinline__ float ex2f(float x) { float y; asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ uint32_t cvtbf(float a, float b) {
  uint32_t r; asm volatile("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(a), "f"(b)); return r; }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d; asm volatile("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(*reinterpret_cast<unsigned long long*>(&d))
      : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)),
        "l"(*reinterpret_cast<unsigned long long*>(&c))); return d; }

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d; asm volatile("add.rn.f32x2 %0, %1, %2;" : "=l"(*reinterpret_cast<unsigned long long*>(&d))
      : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b))); return d; }

// MIX: 0 ex2 x16 | 1 ex2 x16 + ffma2 x8 + cvt x8 | 2 ffma2 x16 |
//      3 the attention kernel's exponential loop over a 128-column row: per
//        pair ffma2 (scale, subtract the max) -> 2 ex2 -> add.f32x2 (row sum)
//        and cvt (pack P); 128 ex2 per iteration, reported per 16 ex2
// KIND of the MMA stream: 0 SS N=128, D alternating between two accumulators
// every 4 MMAs | 1 SS N=128, one accumulator | 2 TS N=128 (A from TMEM) |
// 3 SS N=256 | 4 SS N=64
template <int MIX, bool MMA, int W, int KIND = 0>
__global__ void __launch_bounds__(384, 1) bench(unsigned long long* cyc, unsigned long long* mma_done,
                                                uint32_t* sink, int* status, int zero_operands) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  // Operands: bf16 values in [0.125, 0.25) from a hash of the index (or zeros).
  for (int i = threadIdx.x; i < kOperandBytes / 4; i += blockDim.x) {
    const uint32_t h0 = (static_cast<uint32_t>(i) * 2654435761u) >> 16;
    const uint32_t h1 = (static_cast<uint32_t>(i) * 2246822519u) >> 16;
    reinterpret_cast<uint32_t*>(smem)[i] =
        zero_operands ? 0u : (0x3E00u | (h0 & 0x7Fu)) | ((0x3E00u | (h1 & 0x7Fu)) << 16);
  }
  const uint32_t bar0 = sbase + kOperandBytes;
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + kOperandBytes + 64);
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) { mbar_init(bar0, 1); mbar_init(bar0 + 8, 1); fence_mbarrier_init(); }
  if (warp == 2) { tmem_alloc(smem_u32(slot), 512); tmem_relinquish(); }
  fence_proxy_async_shared();
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(slot);

  if (MMA && warp == 0) {
    const uint32_t leader = (threadIdx.x & 31) == 0 ? 1u : 0u;
    constexpr int kN = KIND == 3 ? 256 : KIND == 4 ? 64 : 128;
    constexpr uint32_t idesc = idesc_f16_f32(128, kN, true, false);
    const uint32_t a_lo = sdesc_lo(sbase, 16), b_lo = sdesc_lo(sbase + 16384, 16);
    // Issue blocks while about four MMAs are queued, so the loop runs at the
    // tensor core's own rate; one commit at the end.
    const unsigned long long m0 = clock64();
    int g = 0;
    for (; g < kMmaGroups; ++g) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (KIND == 2)  // A: 8 TMEM columns of packed bf16 per K-step, at column 256
          umma_f16_ts(tmem, tmem + 256u + i * 8u, b_lo + i * 2u, idesc, 1u, leader);
        else if constexpr (KIND == 0)
          umma_f16_ss(tmem + (g & 1) * 128u, a_lo + i * 2u, b_lo + i * 2u, idesc, 1u, leader);
        else
          umma_f16_ss(tmem, a_lo + i * 2u, b_lo + i * 2u, idesc, 1u, leader);
      }
    }
    umma_commit(bar0, leader);
    bool done = false;
    for (int k = 0; k < (1 << 24) && !done; ++k) done = mbar_try_wait(bar0, 0u);
    if (!done && leader) atomicExch(status, 1);
    // Cycles per MMA over the whole stream (64 = the tensor core's rate at N = 128).
    if (leader) mma_done[blockIdx.x] = (clock64() - m0) * 100ull / (static_cast<unsigned long long>(g) * 4ull);
  } else if (warp >= 4 && warp < 4 + 4 * W) {
    float v[16];
    float2 w2[16];
    for (int i = 0; i < 16; ++i) {
      v[i] = (i + 1) * 1e-3f - 3.f + threadIdx.x * 1e-5f;
      w2[i] = make_float2(v[i], v[i] * 0.5f);
    }
    const float2 c2 = make_float2(0.999f, 1.0001f), d2 = make_float2(1e-7f, -1e-7f);
    uint32_t acc = 0;
    float sc[128];
    for (int i = 0; i < 128; ++i) sc[i] = -0.01f * i - threadIdx.x * 1e-4f;
    const unsigned long long t0 = clock64();
    if constexpr (MIX == 3) {
      float2 a0 = make_float2(0.f, 0.f), a1 = a0;
      const float2 nm = make_float2(-0.5f, -0.5f);
      for (int it = 0; it < ITERS / 8; ++it) {
#pragma unroll
        for (int k = 0; k < 128; k += 2) {
          const float2 x = ffma2(make_float2(sc[k], sc[k + 1]), c2, nm);
          const float2 e = make_float2(ex2f(x.x), ex2f(x.y));
          if ((k >> 1) & 1) a1 = fadd2(a1, e); else a0 = fadd2(a0, e);
          acc ^= cvtbf(e.x, e.y);
        }
        sc[0] += a0.x * 1e-30f;  // a loop-carried use (the asm statements are volatile)
      }
      v[0] = a0.x + a0.y + a1.x + a1.y;
    }
    for (int it = 0; it < (MIX == 3 ? 0 : ITERS); ++it) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (MIX == 0 || MIX == 1) v[i] = ex2f(v[i]) - 1.0f;
        if (MIX == 1 && (i & 1)) { w2[i] = ffma2(w2[i], c2, d2); acc ^= cvtbf(w2[i].x, w2[i].y); }
        if (MIX == 2) w2[i] = ffma2(w2[i], c2, d2);
      }
    }
    const unsigned long long t1 = clock64();
    for (int i = 0; i < 16; ++i) acc ^= __float_as_uint(v[i]) ^ __float_as_uint(w2[i].x) ^ __float_as_uint(w2[i].y);
    sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
    if ((threadIdx.x & 31) == 0) cyc[blockIdx.x * 8 + (warp - 4)] = t1 - t0;
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) { tc_fence_after_sync(); tmem_dealloc(tmem, 512); }
}

template <int MIX, bool MMA, int W, int KIND = 0>
void run(const char* name, int sms, int zero_operands = 0) {
  unsigned long long *dcyc, *dmma; uint32_t* dsink; int* dst;
  cudaMalloc(&dcyc, sizeof(unsigned long long) * sms * 8);
  cudaMalloc(&dmma, sizeof(unsigned long long) * sms);
  cudaMalloc(&dsink, sizeof(uint32_t) * sms * 384);
  cudaMalloc(&dst, 4);
  cudaMemset(dst, 0, 4);
  cudaMemset(dmma, 0, sizeof(unsigned long long) * sms);
  const int smem = 120 * 1024;  // more than half an SM's shared memory: one CTA per SM
  cudaFuncSetAttribute(bench<MIX, MMA, W, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  for (int rep = 0; rep < 2; ++rep)
    bench<MIX, MMA, W, KIND><<<sms, 384, smem>>>(dcyc, dmma, dsink, dst, zero_operands);
  const cudaError_t e = cudaDeviceSynchronize();
  static unsigned long long h[148 * 8], hm[148];
  int hs = 0;
  cudaMemcpy(h, dcyc, sizeof(unsigned long long) * sms * 8, cudaMemcpyDeviceToHost);
  cudaMemcpy(hm, dmma, sizeof(unsigned long long) * sms, cudaMemcpyDeviceToHost);
  cudaMemcpy(&hs, dst, 4, cudaMemcpyDeviceToHost);
  double s = 0;
  for (int b = 0; b < sms; ++b)
    for (int w = 0; w < 4 * W; ++w) s += h[b * 8 + w];
  // A warp's loop time / ITERS is per group of that warp; W warps share a sub-partition.
  const double per_group = W ? s / (sms * 4.0 * W) / ITERS / W : 0.0;
  double mma = 0;
  for (int b = 0; b < sms; ++b) mma += hm[b];
  printf("%-34s W=%d  %7.2f cycles per 16-instruction group per sub-partition;  %6.2f cycles per MMA  (%s, status %d)\n",
         name, W, per_group, MMA ? mma / sms / 100.0 : 0.0, cudaGetErrorString(e), hs);
  cudaFree(dcyc); cudaFree(dmma); cudaFree(dsink); cudaFree(dst);
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  if (sms > 148) sms = 148;
  run<0, true, 0>("MMAs alone", sms);
  run<0, true, 0>("MMAs alone, zero operands", sms, 1);
  run<0, true, 0>("MMAs alone, one SM", 1);
  run<0, true, 0, 1>("MMAs alone, one accumulator", sms);
  run<0, true, 0, 2>("MMAs alone, TS N=128", sms);
  run<0, true, 0, 3>("MMAs alone, SS N=256", sms);
  run<0, true, 0, 4>("MMAs alone, SS N=64", sms);
  run<0, false, 1>("ex2 x16, tensor core idle", sms);
  run<0, true, 1>("ex2 x16, MMAs queued", sms);
  run<0, false, 2>("ex2 x16, tensor core idle", sms);
  run<0, true, 2>("ex2 x16, MMAs queued", sms);
  run<1, false, 1>("softmax mix, tensor core idle", sms);
  run<1, true, 1>("softmax mix, MMAs queued", sms);
  run<1, false, 2>("softmax mix, tensor core idle", sms);
  run<1, true, 2>("softmax mix, MMAs queued", sms);
  run<2, false, 1>("ffma2 x16, tensor core idle", sms);
  run<2, true, 1>("ffma2 x16, MMAs queued", sms);
  run<2, false, 2>("ffma2 x16, tensor core idle", sms);
  run<2, true, 2>("ffma2 x16, MMAs queued", sms);
  run<3, false, 1>("kernel exp loop, tensor core idle", sms);
  run<3, true, 1>("kernel exp loop, MMAs queued", sms);
  run<3, false, 2>("kernel exp loop, tensor core idle", sms);
  run<3, true, 2>("kernel exp loop, MMAs queued", sms);
  return 0;
}
