"""CPU oracle for the attention forward -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this module, and only as the checker or the timed CPU baseline;
the product path (afa_flash_attention_kernels.forward -> libafa_sm100.so) never
calls it.

What it restates: the reference's attention forward, O = softmax(Q K^T * scale) V
per (batch, head) slice, non-causal, no dropout, scale = 1/sqrt(d_head)
(csrc/include/afa_forward_kernel.cuh:83-84 folds log2(e) into that scale and
uses exp2; mathematically the same softmax).  Layout [B, N, H, d].

Beyond the reference (which has neither), ``attention_fp32`` and
``attention_fp64`` also take K/V with their own length and head count
(query head h reads K/V head h // (H // H_kv)), a causal mask aligned to the
bottom-right corner (query row i sees keys j <= i + N_kv - N; a row that sees
no key gives O = 0 and log-sum-exp -inf) and return the log-sum-exp
ln(sum_j exp(scale * q_i . k_j)) per row on request.

Three forms:
* ``attention_fp32``       -- fp32 math on the (fp16/bf16-valued) inputs, the
  "naive torch fp32 softmax(QK^T*scale)V" oracle named by the north star; also
  the timed CPU baseline.  Chunked over (b, h) so N x N scores never
  materialise for all heads at once.
* ``attention_fp64``       -- float64 numpy, used to pin the fp32 oracle.
* ``attention_blockwise``  -- numpy restatement of the reference kernel's own
  blockwise algorithm (afa_forward_kernel.cuh:110-184 with
  afa_softmax.cuh:25-127): B_r x B_c tiles, running max m and sum l, an
  unconditional rescale of l and O per KV block, l summed from fp32 P
  (afa_softmax.cuh:93-105) before P is rounded to the input dtype for the PV
  product (afa_forward_kernel.cuh:166), final O / l (afa_softmax.cuh:107-127)
  and a cast to the input dtype.  Slow (Python loop over tiles); for small
  shapes only.

Parity of this oracle is pinned by tests/test_oracle.py: against float64,
against torch's SDPA math backend, and against golden outputs of the
reference's own CUDA kernel (tests/golden/).
"""

from __future__ import annotations

import math

import numpy as np
import torch

LOG2E = 1.4426950408889634


def default_scale(d_head: int) -> float:
    """1/sqrt(d): the reference's fixed scale (afa_forward_kernel.cuh:83)."""
    return 1.0 / math.sqrt(d_head)


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                   slices=None, max_scores: int = 1 << 26, causal: bool = False,
                   return_lse: bool = False):
    """fp32 softmax(Q K^T * scale) V on CPU (or wherever the inputs live).

    q: [B, N, H, d]; k, v: [B, N_kv, H_kv, d] (H_kv divides H) of any float
    dtype; values are taken exactly and the arithmetic is fp32.  ``slices``:
    optional list of (b, h) pairs; when given, returns [len(slices), N, d] for
    those slices only.  Otherwise returns [B, N, H, d] fp32.  Rows are
    processed in chunks so at most ``max_scores`` fp32 scores exist at once.
    With ``return_lse`` also returns the fp32 log-sum-exp, [B, H, N] (or
    [len(slices), N]).
    """
    B, N, H, d = q.shape
    n_kv, h_kv = k.shape[1], k.shape[2]
    group = H // h_kv
    if scale is None:
        scale = default_scale(d)
    pairs = slices if slices is not None else [(b, h) for b in range(B) for h in range(H)]
    out = torch.empty((len(pairs), N, d), dtype=torch.float32, device=q.device)
    lse = torch.empty((len(pairs), N), dtype=torch.float32, device=q.device)
    rows = max(1, min(N, max_scores // max(n_kv, 1)))
    off = n_kv - N
    keys = torch.arange(n_kv, device=q.device)
    for i, (b, h) in enumerate(pairs):
        qs = q[b, :, h, :].float()
        ks = k[b, :, h // group, :].float()
        vs = v[b, :, h // group, :].float()
        for r0 in range(0, N, rows):
            s = (qs[r0:r0 + rows] @ ks.t()) * scale
            if causal:
                r = torch.arange(r0, min(r0 + rows, N), device=q.device)
                s = s.masked_fill(keys[None, :] > (r[:, None] + off), float("-inf"))
            m = s.amax(dim=-1, keepdim=True)
            m = torch.where(torch.isinf(m), torch.zeros_like(m), m)  # rows that see no key
            p = torch.exp(s - m)
            l = p.sum(dim=-1, keepdim=True)
            out[i, r0:r0 + rows] = torch.where(l > 0, (p @ vs) / l, torch.zeros_like(l))
            lse[i, r0:r0 + rows] = (m + torch.log(l)).squeeze(-1)
    if slices is not None:
        return (out, lse) if return_lse else out
    o = out.view(B, H, N, d).permute(0, 2, 1, 3).contiguous()
    return (o, lse.view(B, H, N)) if return_lse else o


def attention_fp64(q, k, v, scale: float | None = None, causal: bool = False, return_lse: bool = False):
    """float64 numpy softmax(Q K^T * scale) V; q [B, N, H, d], k, v [B, N_kv, H_kv, d]
    (torch or numpy).  Same mask and log-sum-exp conventions as attention_fp32."""
    qn, kn, vn = (np.asarray(t.float().cpu().numpy() if isinstance(t, torch.Tensor) else t, dtype=np.float64)
                  for t in (q, k, v))
    B, N, H, d = qn.shape
    n_kv, h_kv = kn.shape[1], kn.shape[2]
    kn = np.repeat(kn, H // h_kv, axis=2)
    vn = np.repeat(vn, H // h_kv, axis=2)
    if scale is None:
        scale = default_scale(d)
    s = np.einsum("bnhd,bmhd->bhnm", qn, kn) * scale
    if causal:
        mask = np.arange(n_kv)[None, :] > (np.arange(N)[:, None] + (n_kv - N))
        s = np.where(mask[None, None], -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isinf(m), 0.0, m)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        o = np.einsum("bhnm,bmhd->bnhd", np.where(l > 0, p / l, 0.0), vn)
        lse = (m + np.log(l))[..., 0]
    return (o, lse) if return_lse else o


def _round_to(x: np.ndarray, torch_dtype) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch_dtype).float().numpy()


def attention_blockwise(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, B_r: int = 64, B_c: int = 32,
                        scale: float | None = None) -> torch.Tensor:
    """The reference kernel's blockwise online softmax, restated in numpy.

    Per (b, h) and per B_r-row query block (afa_forward_kernel.cuh:31-49):
      for each B_c-column KV block j (:110):
        S = Q K_j^T in fp32 (:137)
        m_next = max(m, rowmax(S))                      (afa_softmax.cuh:25-45)
        alpha = exp2((m - m_next) * c); l *= alpha; O *= alpha   (:47-68, unconditional)
        P = exp2(S * c - m_next * c)                     (:70-91)
        l += rowsum(P)  -- fp32 P                        (:93-105)
        O += round_dtype(P) V_j  in fp32                 (afa_forward_kernel.cuh:166,181)
      O = O / l, rounded to the input dtype              (afa_softmax.cuh:107-127, :186)
    with c = log2(e) / sqrt(d) (afa_forward_kernel.cuh:83-84).
    Requires N % B_r == 0 and N % B_c == 0, as the reference does.
    Returns [B, N, H, d] in the input dtype.
    """
    B, N, H, d = q.shape
    if N % B_r or N % B_c:
        raise ValueError("the reference requires seq_len to be a multiple of B_r and B_c")
    dt = q.dtype
    c = (default_scale(d) if scale is None else scale) * LOG2E
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    out = np.empty((B, N, H, d), dtype=np.float32)
    for b in range(B):
        for h in range(H):
            for r0 in range(0, N, B_r):
                Q = qn[b, r0:r0 + B_r, h, :]
                m = np.full((B_r,), -np.inf, dtype=np.float32)
                l = np.zeros((B_r,), dtype=np.float32)
                O = np.zeros((B_r, d), dtype=np.float32)
                for c0 in range(0, N, B_c):
                    K = kn[b, c0:c0 + B_c, h, :]
                    V = vn[b, c0:c0 + B_c, h, :]
                    S = (Q @ K.T).astype(np.float32)
                    m_next = np.maximum(m, S.max(axis=1))
                    alpha = np.exp2((m - m_next) * c).astype(np.float32)
                    l *= alpha
                    O *= alpha[:, None]
                    m = m_next
                    P = np.exp2(S * c - (m * c)[:, None]).astype(np.float32)
                    l += P.sum(axis=1, dtype=np.float32)
                    O += _round_to(P, dt) @ V
                out[b, r0:r0 + B_r, h, :] = O / l[:, None]
    return torch.from_numpy(out).to(dt)


def error_stats(out: torch.Tensor, ref: torch.Tensor) -> tuple[float, float]:
    """(max-abs, mean-abs) of out - ref in fp32, the metrics of demo.py:61-62."""
    diff = (out.float().cpu() - ref.float().cpu()).abs()
    return float(diff.max()), float(diff.mean())
