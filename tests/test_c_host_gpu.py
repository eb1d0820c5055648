"""The C ABI used from a plain C host program, with no Python or torch in the
process: the program is compiled against include/afa_sm100.h, links
libafa_sm100.so and the CUDA runtime, allocates its buffers with cudaMalloc,
fills Q, K, V from a fixed generator, calls afa_fwd_sm100 (and, for the causal
case, afa_fwd_sm100_noalloc) and writes O to a file.  The test regenerates the
same inputs and checks O against the fp32 oracle within the fp16 tolerances."""

import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_oracle import attention_fp32, error_stats

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "ampere_flash_attention_from_scratch_b200"
CUDA = Path("/usr/local/cuda")

C_SRC = r"""
#include <stdio.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <cuda_runtime.h>
#include "afa_sm100.h"

/* Same generator as the test: element i of tensor `seed` is splitmix64(seed << 32 | i),
   value = ((z >> 40) / 2^24 - 0.5) * 4, rounded to fp16. */
static uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
static void fill(_Float16* h, size_t n, uint64_t seed) {
  for (size_t i = 0; i < n; ++i) {
    uint64_t z = splitmix64((seed << 32) | (uint64_t)i);
    float v = ((float)(z >> 40) / 16777216.0f - 0.5f) * 4.0f;
    h[i] = (_Float16)v; /* IEEE binary16, round to nearest even */
  }
}

int main(int argc, char** argv) {
  const int B = 2, N = 777, H = 4, D = 128, causal = atoi(argv[1]), noalloc = atoi(argv[2]);
  const size_t n = (size_t)B * N * H * D, bytes = n * sizeof(_Float16);
  _Float16 *hq = malloc(bytes), *hk = malloc(bytes), *hv = malloc(bytes), *ho = malloc(bytes);
  fill(hq, n, 1); fill(hk, n, 2); fill(hv, n, 3);
  void *dq, *dk, *dv, *dout; int32_t* dstatus;
  if (cudaMalloc(&dq, bytes) || cudaMalloc(&dk, bytes) || cudaMalloc(&dv, bytes) || cudaMalloc(&dout, bytes) ||
      cudaMalloc((void**)&dstatus, 4)) { fprintf(stderr, "cudaMalloc failed\n"); return 2; }
  cudaMemcpy(dq, hq, bytes, cudaMemcpyHostToDevice);
  cudaMemcpy(dk, hk, bytes, cudaMemcpyHostToDevice);
  cudaMemcpy(dv, hv, bytes, cudaMemcpyHostToDevice);
  cudaMemset(dstatus, 0, 4);
  AfaFwdArgs a;
  memset(&a, 0, sizeof a);
  a.q = dq; a.k = dk; a.v = dv; a.o = dout;
  int64_t s[3] = {(int64_t)N * H * D, (int64_t)H * D, D};
  memcpy(a.q_strides, s, sizeof s); memcpy(a.k_strides, s, sizeof s);
  memcpy(a.v_strides, s, sizeof s); memcpy(a.o_strides, s, sizeof s);
  a.batch = B; a.seq_len = N; a.n_heads = H; a.head_dim = D;
  a.dtype = AFA_DTYPE_FP16; a.status = dstatus; a.causal = causal;
  int rc = noalloc ? afa_fwd_sm100_noalloc(&a, 0) : afa_fwd_sm100(&a, 0);
  if (rc != AFA_OK) { fprintf(stderr, "launch: %s\n", afa_strerror(rc)); return 3; }
  int32_t st = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) { fprintf(stderr, "sync failed\n"); return 4; }
  cudaMemcpy(&st, dstatus, 4, cudaMemcpyDeviceToHost);
  if (st != 0) { fprintf(stderr, "device: %s\n", afa_status_string(st)); return 5; }
  cudaMemcpy(ho, dout, bytes, cudaMemcpyDeviceToHost);
  FILE* f = fopen(argv[3], "wb");
  fwrite(ho, 1, bytes, f);
  fclose(f);
  printf("ok version %d\n", afa_sm100_version());
  return 0;
}
"""


def _fill(n, seed):
    """The C program's generator, vectorised (uint64 arithmetic wraps as in C)."""
    with np.errstate(over="ignore"):
        z = (np.uint64(seed) << np.uint64(32)) | np.arange(n, dtype=np.uint64)
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    v = ((z >> np.uint64(40)).astype(np.float32) / np.float32(16777216.0) - np.float32(0.5)) * np.float32(4.0)
    return torch.from_numpy(v).half()


@pytest.fixture(scope="module")
def c_program(tmp_path_factory):
    d = tmp_path_factory.mktemp("chost")
    src = d / "host.c"
    src.write_text(C_SRC)
    exe = d / "host"
    subprocess.run(["gcc", "-O2", "-std=c11", str(src), "-o", str(exe), f"-I{ROOT / 'include'}",
                    f"-I{CUDA / 'include'}", f"-L{PKG}", "-l:libafa_sm100.so", f"-L{CUDA / 'lib64'}", "-lcudart",
                    f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{CUDA / 'lib64'}"], check=True)
    return exe


@pytest.mark.parametrize("causal,noalloc", [(0, 0), (1, 0), (1, 1)])
def test_plain_c_host(c_program, tmp_path, causal, noalloc):
    out_file = tmp_path / "o.bin"
    r = subprocess.run([str(c_program), str(causal), str(noalloc), str(out_file)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("ok version")
    B, N, H, D = 2, 777, 4, 128
    n = B * N * H * D
    o = torch.from_numpy(np.fromfile(out_file, dtype=np.float16)).view(B, N, H, D)
    q, k, v = (_fill(n, s).view(B, N, H, D) for s in (1, 2, 3))
    ref = attention_fp32(q.cuda(), k.cuda(), v.cuda(), causal=bool(causal))
    mx, mean = error_stats(o, ref)
    assert mx <= 1e-2 and mean <= 1e-3, f"max-abs {mx:.3e} mean-abs {mean:.3e}"
