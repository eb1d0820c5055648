// ref_kernel_shim.cu -- TEST INFRASTRUCTURE ONLY (oracle).
//
// Exposes the reference's own Ampere attention kernel,
// afa::afa_forward_kernel<AFAForwardKernelTraits<cfg>>
// (csrc/include/afa_forward_kernel.cuh:18-202 of the reference), through a
// small C ABI so the parity tests can run it on the same inputs as the sm_100a
// kernel.  This file contains no kernel code of its own: it is compiled by
// oracle/build_ref.py against the reference's headers where they lie, as PTX
// for compute_80 only, so the driver JIT-compiles it for the B200 at load time.
// The launch mirrors csrc/ampere_flash_attention.cu:101-127 of the reference.
#include <cuda_runtime.h>

#include "afa_config.cuh"
#include "afa_forward_kernel.cuh"
#include "afa_kernel_traits.cuh"

namespace {
using afa::AFAForwardKernelConfig;
using afa::AFAForwardKernelTraits;

// The reference's default config: AFAForwardKernelConfig() of afa_py/afa_config.py:33-48.
constexpr AFAForwardKernelConfig kFp16D128{torch::kFloat16, 128, 64, 32, 4, true, true, true, true, true, 2, 2, 2};
// B_r=128, B_c=64, 8 warps (README row 7').
constexpr AFAForwardKernelConfig kFp16D128Wide{torch::kFloat16, 128, 128, 64, 8, true, true, true, true, true, 2, 2, 2};
// Not in the reference's shipped presets; compiled from the same template for cfg5 cross-checks.
constexpr AFAForwardKernelConfig kBf16D64{torch::kBFloat16, 64, 64, 32, 4, true, true, true, true, true, 2, 2, 2};

template <AFAForwardKernelConfig cfg>
int launch(const void* q, const void* k, const void* v, void* o, int B, int N, int H, cudaStream_t st) {
  if (N % cfg.B_r != 0 || N % cfg.B_c != 0) return 1;
  const int64_t d = cfg.d_head;
  afa::AFAForwardParams args{const_cast<void*>(q), const_cast<void*>(k), const_cast<void*>(v), o,
                             static_cast<int64_t>(N) * H * d, static_cast<int64_t>(H) * d, d, N, H,
                             N / cfg.B_r, N / cfg.B_c};
  const int smem = cfg.smem_bytes();
  auto kern = afa::afa_forward_kernel<AFAForwardKernelTraits<cfg>>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(N / cfg.B_r, H, B);
  kern<<<grid, cfg.n_warps * 32, smem, st>>>(args);
  return static_cast<int>(cudaGetLastError());
}
}  // namespace

// config: 0 = fp16 d128 default, 1 = fp16 d128 (128, 64, 8 warps), 2 = bf16 d64.
// Inputs contiguous [B, N, H, d].  Returns 0 on success.
extern "C" int afa_ref_forward(int config, const void* q, const void* k, const void* v, void* o, int B,
                               int N, int H, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (config) {
    case 0: return launch<kFp16D128>(q, k, v, o, B, N, H, st);
    case 1: return launch<kFp16D128Wide>(q, k, v, o, B, N, H, st);
    case 2: return launch<kBf16D64>(q, k, v, o, B, N, H, st);
    default: return 2;
  }
}
