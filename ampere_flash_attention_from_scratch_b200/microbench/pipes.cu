// pipes.cu -- cycles per warp instruction of the softmax's arithmetic on one SM
// sub-partition: ex2.approx (MUFU), cvt.rn.{bf16x2,f16x2}.f32, fma.rn.f32x2,
// scalar fma, 3-input max, and mixes of them (whether two kinds overlap or
// share a pipe).  One CTA per SM with 4, 8 or 16 warps (1, 2 or 4 per
// sub-partition), 16 independent chains per thread, in-kernel clock64.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -o pipes \
//        ampere_flash_attention_from_scratch_b200/microbench/pipes.cu && ./pipes
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>

__device__ __forceinline__ float ex2a(float x) { float y; asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ uint32_t cvtbf(float a, float b) {
  uint32_t r; asm volatile("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(a), "f"(b)); return r; }
__device__ __forceinline__ uint32_t cvth(float a, float b) {
  uint32_t r; asm volatile("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(a), "f"(b)); return r; }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d; asm volatile("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(*reinterpret_cast<unsigned long long*>(&d))
      : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)),
        "l"(*reinterpret_cast<unsigned long long*>(&c))); return d; }
__device__ __forceinline__ float ffma1(float a, float b, float c) { float d; asm volatile("fma.rn.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c)); return d; }
__device__ __forceinline__ float fmax3(float a, float b, float c) { float d; asm volatile("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c)); return d; }

constexpr int ITERS = 2048;

// MODE: 0 ex2 x16 | 1 cvt bf16 x16 | 2 ex2 x16 + cvt x8 | 3 ffma2 x16 | 4 ex2 x16 + ffma2 x16 |
//       5 ffma x16 | 6 ex2 x16 + ffma x16 | 7 max3 x16 | 8 ex2 x16 + max3 x8 | 9 cvt f16 x16 |
//       10 ex2 x16 + cvt f16 x8 | 11 ex2 x16 + ffma2 x8 + cvt x8 (the softmax's mix)
template <int MODE>
__global__ void kern(float seed, unsigned long long* cyc, uint32_t* sink) {
  float v[16];
  float2 w[16];
  for (int i = 0; i < 16; ++i) { v[i] = seed * (i + 1) * 1e-3f - 3.f + threadIdx.x * 1e-5f; w[i] = make_float2(v[i], v[i] * 0.5f); }
  const float2 c2 = make_float2(0.999f, 1.0001f), d2 = make_float2(1e-7f, -1e-7f);
  uint32_t acc = 0;
  __syncthreads();
  const unsigned long long t0 = clock64();
  for (int it = 0; it < ITERS; ++it) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (MODE == 0 || MODE == 2 || MODE == 4 || MODE == 6 || MODE == 8 || MODE == 10 || MODE == 11) v[i] = ex2a(v[i]) - 1.0f;
      if (MODE == 1) acc ^= cvtbf(v[i], v[(i + 1) & 15]), v[i] += 1e-7f;
      if (MODE == 9) acc ^= cvth(v[i], v[(i + 1) & 15]), v[i] += 1e-7f;
      if ((MODE == 2 || MODE == 11) && (i & 1)) acc ^= cvtbf(w[i].x, w[i].y);
      if (MODE == 10 && (i & 1)) acc ^= cvth(w[i].x, w[i].y);
      if (MODE == 3 || MODE == 4) w[i] = ffma2(w[i], c2, d2);
      if (MODE == 11 && (i & 1)) w[i] = ffma2(w[i], c2, d2);
      if (MODE == 5 || MODE == 6) w[i].x = ffma1(w[i].x, 0.999f, 1e-7f);
      if (MODE == 7) w[i].x = fmax3(w[i].x, w[(i + 1) & 15].y, v[i]) * 0.999f;
      if (MODE == 8 && (i & 1)) w[i].x = fmax3(w[i].x, w[(i + 1) & 15].y, 0.f);
    }
  }
  const unsigned long long t1 = clock64();
  for (int i = 0; i < 16; ++i) acc ^= __float_as_uint(v[i]) ^ __float_as_uint(w[i].x) ^ __float_as_uint(w[i].y);
  sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
  if ((threadIdx.x & 31) == 0) cyc[blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32] = t1 - t0;
}

template <int MODE>
void run(const char* name, int warps, unsigned long long* dcyc, uint32_t* dsink, int sms) {
  kern<MODE><<<sms, warps * 32>>>(1.0f, dcyc, dsink);
  kern<MODE><<<sms, warps * 32>>>(1.0f, dcyc, dsink);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) { printf("%s: %s\n", name, cudaGetErrorString(e)); return; }
  static unsigned long long h[148 * 32];
  cudaMemcpy(h, dcyc, sizeof(unsigned long long) * sms * warps, cudaMemcpyDeviceToHost);
  double s = 0; for (int i = 0; i < sms * warps; ++i) s += h[i];
  const double cyc_per_iter = s / (sms * warps) / ITERS;
  printf("%-32s warps/CTA %2d  per sub-partition: %6.2f cycles per 16-instruction group\n", name, warps,
         cyc_per_iter / (warps / 4.0));
}

int main() {
  int sms = 0; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  if (sms > 148) sms = 148;
  unsigned long long* dcyc; uint32_t* dsink;
  cudaMalloc(&dcyc, sizeof(unsigned long long) * sms * 32);
  cudaMalloc(&dsink, sizeof(uint32_t) * sms * 1024);
  for (int warps : {4, 8, 16}) {
    run<0>("ex2 x16", warps, dcyc, dsink, sms);
    run<1>("cvt.bf16x2 x16", warps, dcyc, dsink, sms);
    run<9>("cvt.f16x2 x16", warps, dcyc, dsink, sms);
    run<2>("ex2 x16 + cvt.bf16x2 x8", warps, dcyc, dsink, sms);
    run<10>("ex2 x16 + cvt.f16x2 x8", warps, dcyc, dsink, sms);
    run<3>("ffma2 x16", warps, dcyc, dsink, sms);
    run<4>("ex2 x16 + ffma2 x16", warps, dcyc, dsink, sms);
    run<5>("ffma x16", warps, dcyc, dsink, sms);
    run<6>("ex2 x16 + ffma x16", warps, dcyc, dsink, sms);
    run<7>("max3 x16", warps, dcyc, dsink, sms);
    run<8>("ex2 x16 + max3 x8", warps, dcyc, dsink, sms);
    run<11>("ex2 x16 + ffma2 x8 + cvt x8", warps, dcyc, dsink, sms);
  }
  cudaFree(dcyc); cudaFree(dsink);
  return 0;
}
