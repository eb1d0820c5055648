// afa_fwd_kernel.cuh -- Blackwell (sm_100a) FlashAttention forward kernel.
//
// Computes O = softmax(Q K^T * scale) V for one (batch, head) slice per work
// item, fp16/bf16 in, fp32 accumulate, fp16/bf16 out.  The non-causal,
// equal-shape case is the reference's afa_forward_kernel
// (csrc/include/afa_forward_kernel.cuh:18-202); beyond it the kernel takes a
// key/value length different from the query length, grouped K/V heads (query
// head h reads K/V head h / kv_group), an optional causal mask aligned to the
// bottom-right corner (query row i sees keys j <= i + seq_len_kv - seq_len,
// the FlashAttention convention) and an optional fp32 log-sum-exp output.
// Re-designed for sm_100a:
//
//   * persistent grid (one CTA per SM) walking work items (b, h, q-pair);
//     a q-pair is 256 query rows = two 128-row Q tiles.  Items are dealt
//     round-robin, or -- for the causal kernel given scheduler words --
//     claimed dynamically by the producer and passed to the other warps
//     through a small ring in shared memory (WorkQueue);
//   * warp 0      : TMA producer.  Q0/Q1 once per work item and K_j, V_j
//                   into a kStages-deep ring of 128-row slots (SWIZZLE_128B);
//                   an unmasked item's first K tile goes ahead of its Q tiles;
//   * warp 1      : MMA issuer (the warp computes operands, lane 0 issues).
//                   S_i = Q_i K_j^T and O_i += P_i V_j with tcgen05.mma,
//                   completion via tcgen05.commit -> mbarrier;
//   * warp 2      : TMEM allocator (512 columns: S0 | S1 | O0 | O1);
//   * warps 4-7   : softmax warpgroup 0 (Q tile 0), warps 8-11: warpgroup 1.
//                   One thread owns one query row (one TMEM lane): row max,
//                   exp2, row sum and the final 1/l need no shuffles.  P is
//                   written back into TMEM over S and consumed from TMEM by
//                   the PV MMA.  O is rescaled in TMEM only when a row max
//                   grows by more than 2^8 (conditional rescaling).
//
// The MMA issue order  PV0(j-1), S0(j), PV1(j-1), S1(j)  lets warpgroup 0
// run its softmax on S0(j) while the tensor core works on PV1(j-1) and S1(j),
// and vice versa (ping-pong of the two Q tiles).  The order runs on across
// work items (except in the causal kernel at head_dim 128): the next item's
// S0(0) goes between the current item's last PV0 and PV1.
//
// Numerics follow the reference (csrc/include/afa_softmax.cuh:12-127,
// afa_forward_kernel.cuh:83-184): exp2 with log2(e) folded into the scale,
// the row sum l accumulated from fp32 P before P is rounded to the input type
// for the PV product, fp32 accumulation, final O / l in fp32.
//
// Every mbarrier wait is bounded (globaltimer deadline): on expiry the kernel
// records AFA_DEV_TIMEOUT_BASE + site in the status word, raises a CTA-wide
// abort flag and every role returns (the producer first waits, bounded, for
// the loads it still has in flight), so a bug cannot hang the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100_ptx.cuh"

#ifndef AFA_DEV_TIMEOUT_BASE
#define AFA_DEV_TIMEOUT_BASE 0x100
#endif

namespace afa100 {

// Kernel parameters (passed as __grid_constant__).  Built by the host
// launcher in afa_fwd_sm100.cu; replaces AFAForwardParams
// (csrc/include/afa_config.cuh:7-34).
struct FwdParams {
  // 4-D tensor maps, dims ordered by increasing stride: (head_dim, seq, head,
  // batch) when bit t of seq_inner_mask is set, else (head_dim, head, seq,
  // batch).  Box: 64 head_dim elements (128 bytes) x 128 rows, SWIZZLE_128B.
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  // O for TMA stores (correction warpgroup, or AFA_O_TMA_STORE): box 64
  // head_dim elements x 32 rows, SWIZZLE_128B.
  CUtensorMap tm_o;
  unsigned seq_inner_mask;  // bit 0: q, bit 1: k, bit 2: v, bit 3: o
  void* o;
  long long o_sb, o_sn, o_sh;  // element strides of O (head_dim stride is 1)
  int seq_len;     // query rows
  int seq_len_kv;  // key/value rows
  int n_heads;     // query heads
  int kv_group;    // query heads per K/V head
  int n_q_pairs;   // ceil(seq_len / 256)
  int n_kv;        // ceil(seq_len_kv / 128)
  int n_work;      // batch * n_heads * n_q_pairs
  int causal_off;  // seq_len_kv - seq_len: query row i sees keys j <= i + causal_off
  // Division by n_q_pairs and by n_heads as a multiply and shift (see
  // DivMagic): floor(x / d) = (x * mul) >> shift for 0 <= x < 2^31.
  unsigned long long qp_mul, h_mul;
  int qp_shift, h_shift;
  float* lse;      // optional [batch, n_heads, seq_len] fp32 log-sum-exp (natural log)
  int* sched;      // optional scheduler words [2] (causal kernel): 0 at rest; null = static schedule
  float scale_log2;  // scale * log2(e)
  int* status;
  unsigned long long timeout_ns;
  unsigned test_flags;  // bit 0: the producer issues no loads; bit 1: the MMA issuer issues nothing
                        // (both exercise the timeout path; bit 1 with loads in flight);
                        // bit 2: the last CTA leaves the scheduler words non-zero
};

// Bounded-wait sites, reported as AFA_DEV_TIMEOUT_BASE + site.
enum WaitSite : int {
  kSiteLoadQEmpty = 1,
  kSiteLoadKVEmpty = 2,
  kSiteMmaQFull = 3,
  kSiteMmaKFull = 4,
  kSiteMmaVFull = 5,
  kSiteMmaP0 = 6,
  kSiteMmaP1 = 7,
  kSiteSoftmaxS = 8,
  kSiteSoftmaxO = 9,
  kSiteMmaDrain = 10,
  kSiteLoadItem = 11,  // producer waiting for a free slot of the work-item ring
  kSiteReadItem = 12,  // MMA / softmax warps waiting for the next claimed work item
  kSiteCorrAlpha = 13, // correction warp waiting for a softmax warp's row scale factors
  kSiteCorrStats = 14, // correction warp waiting for a softmax warp's final row sums
  kSiteMmaOFree = 15,  // MMA waiting for the previous item's O to be read out
};

// Compile-time layout of one kernel instance.
// With AFA_CORRECTION_WG set, a fourth warpgroup (warps 12-15, one per TMEM
// lane quadrant) takes the correction role off the softmax warpgroups: it
// rescales O in TMEM when a softmax warp reports a grown row maximum, and runs
// the epilogue (O * 1/l, staged through shared memory, TMA-stored), so each
// softmax warpgroup moves on to the next work item as soon as its last P is
// handed over.
#ifndef AFA_CORRECTION_WG
#define AFA_CORRECTION_WG 0
#endif
#ifndef AFA_O_TMA_STORE
#define AFA_O_TMA_STORE 1
#endif

template <int kD, bool kBF16, int kStages>
struct FwdLayout {
  static_assert(kD == 64 || kD == 128, "head_dim must be 64 or 128");
  static constexpr bool kCorr = AFA_CORRECTION_WG != 0;
  // The softmax warps' epilogue writes O through a swizzled shared-memory tile
  // and TMA stores (whole 128-byte lines) instead of one 16-byte store per row
  // and lane.
  static constexpr bool kOTma = AFA_O_TMA_STORE != 0 && !kCorr;
  static constexpr int kBM = 128;  // query rows per Q tile (= TMEM lanes)
  static constexpr int kBN = 128;  // key/value rows per K/V tile
  static constexpr int kAtoms = kD / 64;               // 128-byte swizzle atoms along head_dim
  static constexpr uint32_t kAtomBytes = 128u * 128u;  // one TMA box: 128 rows x 128 bytes
  static constexpr uint32_t kTileBytes = kAtoms * kAtomBytes;
  static constexpr uint32_t kOffQ = 0;  // Q0, Q1
  static constexpr uint32_t kOffKV = 2 * kTileBytes;
  // Correction warpgroup only: per warp a 4 KB staging tile of O (32 rows x
  // 64 head_dim elements, 128-byte swizzled for the TMA store), the softmax
  // warps' reference maxima before / after the current tile [2][128] and
  // final (l, m) per row [2 items][2][128].
  static constexpr uint32_t kStageBytes = 32u * 128u;
  static constexpr uint32_t kOffStage = kOffKV + kStages * kTileBytes;
  static constexpr uint32_t kStageTiles = kCorr ? 4u : (kOTma ? 8u : 0u);  // one per epilogue warp
  static constexpr uint32_t kOffAlpha = kOffStage + kStageTiles * kStageBytes;
  static constexpr uint32_t kOffStats = kOffAlpha + (kCorr ? 2u * 128u * 8u : 0u);
  static constexpr uint32_t kOffBar = kOffStats + (kCorr ? 2u * 2u * 128u * 8u : 0u);
  // mbarrier indices
  // Each Q tile has its own full/empty pair, so the next work item's Q0 loads
  // as soon as the current item's last S0 is issued.
  static constexpr int kBarQFull = 0;                    // [2]
  static constexpr int kBarQEmpty = 2;                   // [2]
  static constexpr int kBarKVFull = 4;                   // [kStages]
  static constexpr int kBarKVEmpty = 4 + kStages;        // [kStages]
  static constexpr int kBarSFull = 4 + 2 * kStages;      // [2]
  // P is handed to the PV MMA in kPChunks column chunks, one barrier each, so
  // the tensor core starts O += P V on the first chunk while the softmax
  // warpgroup is still computing the rest.
#ifndef AFA_P_CHUNKS
#define AFA_P_CHUNKS 2
#endif
  static constexpr int kPChunks = AFA_P_CHUNKS;
  static constexpr int kSColsPerChunk = kBN / kPChunks;       // S columns per chunk (even split)
  static constexpr int kPColsPerChunk = kSColsPerChunk / 2;   // TMEM columns of packed P
  static constexpr int kPvStepsPerChunk = kSColsPerChunk / 16;  // MMA K-steps per chunk
  // Chunk c covers S columns [chunk_begin(c), chunk_begin(c + 1)).  With two
  // chunks the split may be uneven (kPSplit): a short last chunk shortens the
  // PV that stands between the last hand-off and the next S on the critical path.
  // At head_dim 64 the PV MMAs (N = 64) are issue-bound (~48 cycles each for
  // 32 cycles of work), so a 32-column last chunk (2 MMAs instead of 4) pays
  // there; at 128 the even split is as fast.
#ifndef AFA_P_SPLIT
#define AFA_P_SPLIT 64
#endif
#ifndef AFA_P_SPLIT_D64
#define AFA_P_SPLIT_D64 96
#endif
  static constexpr int kPSplit = kD == 64 ? AFA_P_SPLIT_D64 : AFA_P_SPLIT;
  static_assert(kPChunks != 2 || (kPSplit % 32 == 0 && kPSplit > 0 && kPSplit < kBN),
                "the chunk split must fall on a 32-column boundary (16 packed P columns)");
  __host__ __device__ static constexpr int chunk_begin(int c) {
    return kPChunks == 2 ? (c == 0 ? 0 : c == 1 ? kPSplit : kBN) : c * kSColsPerChunk;
  }
  static constexpr int kBarPReady = kBarSFull + 2;       // [2][kPChunks]
  static constexpr int kBarOFinal = kBarPReady + 2 * kPChunks;  // [2]
  static constexpr int kBarMmaDrain = kBarOFinal + 2;
  // Dynamic schedule: ring of kItemSlots claimed work items (producer -> MMA
  // warp and the 8 softmax warps).
  static constexpr int kItemSlots = 4;
  static constexpr int kBarItemFull = kBarMmaDrain + 1;           // [kItemSlots]
  static constexpr int kBarItemEmpty = kBarItemFull + kItemSlots;  // [kItemSlots]
  static constexpr uint32_t kItemReaders = 1 + 8 + (kCorr ? 4 : 0);  // MMA, softmax (+ correction) warps
  // Correction warpgroup only: alpha ready [wg][quadrant], (l, m) ready
  // [wg][quadrant] (one arrival each), O read out [wg] (one arrival per
  // correction warp).  P chunk 0's barrier then also waits for the correction
  // warps (the O rescale precedes the PV that accumulates into O).
  static constexpr int kBarAlpha = kBarItemEmpty + kItemSlots;
  static constexpr int kBarStats = kBarAlpha + (kCorr ? 8 : 0);
  static constexpr int kBarOFree = kBarStats + (kCorr ? 8 : 0);
  static constexpr int kNumBars = kBarOFree + (kCorr ? 2 : 0);
  static constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
  static constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
  static constexpr uint32_t kOffItems = kOffAbort + 4;            // int[kItemSlots]
  static constexpr uint32_t kSmemUsed = kOffItems + 4 * kItemSlots;
  static constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // slack for 1024-byte alignment
  static constexpr int kThreads = kCorr ? 512 : 384;
  static constexpr int kSoftmaxThreads = 128;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColO = 256;  // O0 at 256, O1 at 256 + kD
  // Register split: launched at kLaunchRegs per thread (1 CTA/SM); the
  // producer warpgroup (and the correction warpgroup) drop to kProducerRegs
  // (kCorrRegs), the two softmax warpgroups rise to kSoftmaxRegs.
  // 384 threads: 128 * (72 + 216 + 216) == 384 * 168;
  // 512 threads: 128 * (40 + 208 + 208 + 56) == 512 * 128 (no spills; the
  // softmax warps spill below 208, the correction warps below 56).
#ifndef AFA_CORR_SPLIT_PRODUCER
#define AFA_CORR_SPLIT_PRODUCER 40
#endif
#ifndef AFA_CORR_SPLIT_CORR
#define AFA_CORR_SPLIT_CORR 56
#endif
#ifndef AFA_CORR_SPLIT_SOFTMAX
#define AFA_CORR_SPLIT_SOFTMAX 208
#endif
  static constexpr int kLaunchRegs = kCorr ? 128 : 168;
  static constexpr int kProducerRegs = kCorr ? AFA_CORR_SPLIT_PRODUCER : 72;
  static constexpr int kCorrRegs = AFA_CORR_SPLIT_CORR;
  static constexpr int kSoftmaxRegs = kCorr ? AFA_CORR_SPLIT_SOFTMAX : 216;
  static_assert(kProducerRegs + 2 * kSoftmaxRegs + (kCorr ? kCorrRegs : 0) <= (kThreads / 128) * kLaunchRegs,
                "register split too large");
  // Share of exp2 evaluations moved from the MUFU unit to the FMA pipe: in
  // every group of 8 consecutive column pairs, kEmuPairs evenly spaced pairs
  // use the polynomial (0 by default: every share measured so far was slower).  At head_dim 128 the MUFU work per K/V tile equals the MMA
  // work; at 64 it is twice the MMA work.
#ifndef AFA_EXP_EMU_PAIRS_D128
#define AFA_EXP_EMU_PAIRS_D128 0
#endif
#ifndef AFA_EXP_EMU_PAIRS_D64
#define AFA_EXP_EMU_PAIRS_D64 0
#endif
  static constexpr int kEmuPairs = kD == 128 ? AFA_EXP_EMU_PAIRS_D128 : AFA_EXP_EMU_PAIRS_D64;
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
};

// Bounded mbarrier waits shared by all roles of a CTA.
struct CtaSync {
  volatile int* abort_flag;
  int* status;
  unsigned long long timeout_ns;

  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, int site) const {
    if (mbar_try_wait(bar, parity)) return true;
    return wait_slow(bar, parity, site, true);
  }

  // Records an error code in the status word.  The word may be device memory
  // or mapped page-locked host memory (a host can then read it without
  // synchronising), so it is written with plain stores, not an atomic: when
  // several waits run out, one of their codes remains.
  __device__ __forceinline__ void report(int code) const {
    if (status == nullptr) return;
    volatile int* s = status;
    if (*s == 0) *s = code;
    __threadfence_system();
  }

  // honour_abort = false is used by teardown drains, which must run to the end.
  // Waiting threads are suspended by the hardware between checks (up to
  // kSuspendNs each), so idle warps do not take issue slots from the warps
  // that share their SM sub-partition.
  __device__ __forceinline__ bool wait_slow(uint32_t bar, uint32_t parity, int site,
                                            bool honour_abort) const {
    constexpr uint32_t kSuspendNs = 200000;  // 0.2 ms per suspended check
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      if (mbar_try_wait_suspend(bar, parity, kSuspendNs)) return true;
      if (honour_abort && *abort_flag) return false;
      const uint64_t dt = globaltimer_ns() - t0;
      if (dt > timeout_ns || it > (1u << 30)) {
        *abort_flag = 1;
        report(AFA_DEV_TIMEOUT_BASE + site);
        return false;
      }
    }
  }
};

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// 2^x for two values on the FMA/ALU pipes instead of the MUFU unit.
// Cody-Waite style split x = j + f, j = rint(x) (obtained by adding and
// subtracting 1.5 * 2^23), |f| <= 1/2; 2^f by a degree-3 polynomial whose
// coefficients are a relative-error minimax fit on [-1/2, 1/2] made for this
// kernel (Remez exchange; max relative error 7.2e-5, 1.4e-4 after fp32
// rounding over x in [-126, 8]); 2^j is added to the exponent field.  Inputs
// are clamped to >= -126 so the exponent never wraps (2^-126 ~ 1e-38, zero
// after rounding P to fp16/bf16); inputs never exceed +8 here (conditional
// rescaling bounds x = s*c - m_ref by 8).
__device__ __forceinline__ float2 exp2_fma_pipe2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC0 = 0.99992806f, kC1 = 0.69326097f, kC2 = 0.24261113f, kC3 = 0.05517167f;
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 j = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);
  float2 q = __ffma2_rn(f, make_float2(kC3, kC3), make_float2(kC2, kC2));
  q = __ffma2_rn(q, f, make_float2(kC1, kC1));
  q = __ffma2_rn(q, f, make_float2(kC0, kC0));
  float2 r;
  r.x = __int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23));
  r.y = __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23));
  return r;
}

// Work item w -> (q-pair, head, batch).  Q-pairs of one head are adjacent in
// the order, so the CTAs working at one time share the K/V of a few heads in
// L2.  With a causal mask, q-pairs run from the last (longest) to the first,
// so the round-robin assignment hands out long items first.
// Division of a non-negative int below 2^31 by an invariant divisor d >= 1
// (the round-up method of Granlund and Montgomery, "Division by invariant
// integers using multiplication", 1994): with l = ceil(log2 d), p = 31 + l and
// m = ceil(2^p / d) (at most 2^32), floor(x / d) = floor(x * m / 2^p) for every
// 0 <= x < 2^31, since x * (m - 2^p / d) / 2^p < 2^31 / 2^p <= 1 / d.
struct DivMagic {
  unsigned long long mul;
  int shift;
  __host__ __device__ static DivMagic make(int d) {
    int l = 0;
    while ((1ll << l) < d) ++l;
    const int sh = 31 + l;
    return DivMagic{((1ull << sh) + static_cast<unsigned long long>(d) - 1ull) / static_cast<unsigned long long>(d), sh};
  }
};

__device__ __forceinline__ int div_magic(int x, unsigned long long mul, int shift) {
  return static_cast<int>((static_cast<unsigned long long>(static_cast<unsigned>(x)) * mul) >> shift);
}

template <bool kCausal>
__device__ __forceinline__ void decode_work(const FwdParams& p, int w, int& qp, int& h, int& b) {
  const int bh = div_magic(w, p.qp_mul, p.qp_shift);
  qp = w - bh * p.n_q_pairs;
  if (kCausal) qp = p.n_q_pairs - 1 - qp;
  b = div_magic(bh, p.h_mul, p.h_shift);
  h = bh - b * p.n_heads;
}

// The work items a CTA processes, in order.  Static: blockIdx.x, then every
// gridDim.x-th item.  Dynamic (the causal kernel given scheduler words): the
// producer claims the next item with atomicAdd on sched[0] and publishes it in
// a ring of kItemSlots shared-memory slots, which the MMA warp and the softmax
// warps read in the same order; items of very different length then even out
// across SMs while consecutive items (the same head's K/V, in L2) still run at
// the same time.  After its last claim each CTA counts itself on sched[1]; the
// last one returns both words to 0 for the next launch.
template <int kSlots>
struct WorkQueue {
  int* sched;             // null: static schedule
  volatile int* slots;    // [kSlots]
  uint32_t full0, empty0; // item_full / item_empty barriers
  int n_work;
  bool keep_words;        // test only: the last CTA does not reset the words
  static constexpr int kDone = -1;   // no more items
  static constexpr int kAbort = -2;  // a bounded wait ran out

  __device__ __forceinline__ bool dynamic() const { return sched != nullptr; }

  // Producer (whole warp, converged): item number `it` of this CTA.
  __device__ __forceinline__ int claim(uint32_t it, const CtaSync& sy, int site) const {
    if (!dynamic()) {
      const int w = static_cast<int>(blockIdx.x + it * gridDim.x);
      return w < n_work ? w : kDone;
    }
    const uint32_t slot = it % kSlots, ph = (it / kSlots) & 1u;
    if (!sy.wait(empty0 + 8u * slot, ph ^ 1u, site)) return kAbort;
    int w = 0;
    if ((threadIdx.x & 31u) == 0u) {
      w = atomicAdd(sched, 1);
      if (w >= n_work) w = kDone;
      slots[slot] = w;
      mbar_arrive(full0 + 8u * slot);  // release: the slot write is visible to the readers
    }
    return __shfl_sync(0xffffffffu, w, 0);
  }

  // Readers (whole warp, converged): the same sequence.
  __device__ __forceinline__ int next(uint32_t it, const CtaSync& sy, int site) const {
    if (!dynamic()) {
      const int w = static_cast<int>(blockIdx.x + it * gridDim.x);
      return w < n_work ? w : kDone;
    }
    const uint32_t slot = it % kSlots, ph = (it / kSlots) & 1u;
    if (!sy.wait(full0 + 8u * slot, ph, site)) return kAbort;
    const int w = slots[slot];
    __syncwarp();
    if ((threadIdx.x & 31u) == 0u) mbar_arrive(empty0 + 8u * slot);
    return w;
  }

  // Producer, after its last claim (or an abort): count this CTA; the last
  // CTA resets the words.  Every claim of every CTA precedes its count.
  __device__ __forceinline__ void finish() const {
    if (!dynamic() || (threadIdx.x & 31u) != 0u) return;
    __threadfence();
    if (atomicAdd(sched + 1, 1) == static_cast<int>(gridDim.x) - 1 && !keep_words) {
      atomicExch(sched, 0);
      atomicExch(sched + 1, 0);
    }
  }
};

// K/V tiles that Q tile t (0 or 1) of q-pair qp must visit: all of them, or
// under the causal mask those up to the last key its last query row sees
// (at least one, so a tile whose rows see no key still finishes with O = 0).
// kv_tiles(p, qp, 0) <= kv_tiles(p, qp, 1).
template <bool kCausal>
__device__ __forceinline__ int kv_tiles(const FwdParams& p, int qp, int t) {
  if (!kCausal) return p.n_kv;
  const int last_row = min(qp * 256 + t * 128 + 127, p.seq_len - 1);
  const int last_key = last_row + p.causal_off;
  if (last_key < 0) return 1;
  return min(last_key / 128 + 1, p.n_kv);
}

// ---------------------------------------------------------------------------
// Role: TMA producer (one thread)
// ---------------------------------------------------------------------------
template <int kD, bool kBF16, int kStages, bool kCausal>
__device__ __forceinline__ void role_load(const FwdParams& p, uint32_t sbase, uint32_t bar0,
                                          const CtaSync& sy, const WorkQueue<4>& wq) {
  using L = FwdLayout<kD, kBF16, kStages>;
  auto bar = [&](int i) { return bar0 + 8u * static_cast<uint32_t>(i); };
  const uint64_t pol_kv = l2_policy_evict_last();
  const uint64_t pol_q = l2_policy_evict_first();
  // The whole warp runs this role in converged control flow; lane 0 issues.
  const bool leader = (threadIdx.x & 31u) == 0u;
  uint32_t kv_cnt = 0, q_cnt[2] = {0u, 0u};
  uint32_t it = 0;
  bool ok = true;
  if (p.test_flags & 1u) {  // nothing is loaded: the consumers' bounded waits run out
    wq.finish();
    return;
  }
  for (;; ++it) {
    const int w = wq.claim(it, sy, kSiteLoadItem);
    if (w == wq.kAbort) { ok = false; break; }
    if (w < 0) break;
    int qp, h, b;
    decode_work<kCausal>(p, w, qp, h, b);
    const int h_kv = p.kv_group == 1 ? h : h / p.kv_group;
    const int n_tiles = kv_tiles<kCausal>(p, qp, 1);
    if constexpr (!kCausal) {
      // Unmasked items load K_0, Q0, V_0, Q1, K_1, V_1, ...: K_0 needs only a
      // ring slot, which the previous item freed a tile earlier, while Q1's
      // buffer frees only once that item's last S1 has run, so the first K
      // tile's DRAM latency overlaps the end of the previous item.  (Causal
      // items keep Q first: their Q tile 0 finishes early and frees its buffer
      // before the ring slot frees.)  The ring order is the same either way.
      auto load_q = [&](int t) -> bool {
        if (!sy.wait(bar(L::kBarQEmpty + t), (it & 1u) ^ 1u, kSiteLoadQEmpty)) return false;
        if (leader) mbar_arrive_expect_tx(bar(L::kBarQFull + t), L::kTileBytes);
        const bool si = (p.seq_inner_mask & 1u) != 0u;
#pragma unroll
        for (int a = 0; a < L::kAtoms; ++a) {
          const int row0 = qp * 256 + t * 128;
          if (leader)
            tma_load_4d(sbase + L::kOffQ + t * L::kTileBytes + a * L::kAtomBytes, &p.tm_q,
                        bar(L::kBarQFull + t), a * 64, si ? row0 : h, si ? h : row0, b, pol_q);
        }
        ++q_cnt[t];
        return true;
      };
      auto load_kv = [&](int j, int kv) -> bool {
        const uint32_t slot = kv_cnt % kStages;
        const uint32_t ph = (kv_cnt / kStages) & 1u;
        if (!sy.wait(bar(L::kBarKVEmpty + slot), ph ^ 1u, kSiteLoadKVEmpty)) return false;
        if (leader) mbar_arrive_expect_tx(bar(L::kBarKVFull + slot), L::kTileBytes);
        const CUtensorMap* map = kv ? &p.tm_v : &p.tm_k;
        const bool si = (p.seq_inner_mask & (kv ? 4u : 2u)) != 0u;
#pragma unroll
        for (int a = 0; a < L::kAtoms; ++a) {
          if (leader)
            tma_load_4d(sbase + L::kOffKV + slot * L::kTileBytes + a * L::kAtomBytes, map,
                        bar(L::kBarKVFull + slot), a * 64, si ? j * 128 : h_kv, si ? h_kv : j * 128, b, pol_kv);
        }
        ++kv_cnt;
        return true;
      };
      ok = load_kv(0, 0) && load_q(0) && load_kv(0, 1) && load_q(1);
      for (int j = 1; j < n_tiles && ok; ++j) ok = load_kv(j, 0) && load_kv(j, 1);
      if (!ok) break;
    } else {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (!sy.wait(bar(L::kBarQEmpty + t), (it & 1u) ^ 1u, kSiteLoadQEmpty)) { ok = false; break; }
        if (leader) mbar_arrive_expect_tx(bar(L::kBarQFull + t), L::kTileBytes);
#pragma unroll
        for (int a = 0; a < L::kAtoms; ++a) {
          const int row0 = qp * 256 + t * 128;
          const bool si = (p.seq_inner_mask & 1u) != 0u;
          if (leader)
            tma_load_4d(sbase + L::kOffQ + t * L::kTileBytes + a * L::kAtomBytes, &p.tm_q,
                        bar(L::kBarQFull + t), a * 64, si ? row0 : h, si ? h : row0, b, pol_q);
        }
        ++q_cnt[t];
      }
      if (!ok) break;
      for (int j = 0; j < n_tiles && ok; ++j) {
#pragma unroll
        for (int kv = 0; kv < 2; ++kv) {
          const uint32_t slot = kv_cnt % kStages;
          const uint32_t ph = (kv_cnt / kStages) & 1u;
          if (!sy.wait(bar(L::kBarKVEmpty + slot), ph ^ 1u, kSiteLoadKVEmpty)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(bar(L::kBarKVFull + slot), L::kTileBytes);
          const CUtensorMap* map = kv ? &p.tm_v : &p.tm_k;
          const bool si = (p.seq_inner_mask & (kv ? 4u : 2u)) != 0u;
          const int row0 = j * 128;
#pragma unroll
          for (int a = 0; a < L::kAtoms; ++a) {
            if (leader)
              tma_load_4d(sbase + L::kOffKV + slot * L::kTileBytes + a * L::kAtomBytes, map,
                          bar(L::kBarKVFull + slot), a * 64, si ? row0 : h_kv, si ? h_kv : row0, b,
                          pol_kv);
          }
          ++kv_cnt;
        }
      }
      if (!ok) break;
    }
  }
  wq.finish();
  if (ok) return;
  // Aborted: before the CTA may exit, wait (bounded, not cut short by the
  // abort flag) until the loads still in flight have landed -- the last
  // kStages K/V loads and the last Q load.  Phases that already completed
  // return at once.
  const uint32_t first = kv_cnt > static_cast<uint32_t>(kStages) ? kv_cnt - kStages : 0u;
  for (uint32_t n = first; n < kv_cnt; ++n) {
    const uint32_t fb = bar(L::kBarKVFull + static_cast<int>(n % kStages));
    if (!mbar_try_wait(fb, (n / kStages) & 1u)) sy.wait_slow(fb, (n / kStages) & 1u, kSiteLoadKVEmpty, false);
  }
  for (int t = 0; t < 2; ++t)
    if (q_cnt[t] > 0 && !mbar_try_wait(bar(L::kBarQFull + t), (q_cnt[t] - 1u) & 1u))
      sy.wait_slow(bar(L::kBarQFull + t), (q_cnt[t] - 1u) & 1u, kSiteLoadQEmpty, false);
}

// ---------------------------------------------------------------------------
// Role: MMA issuer (one thread)
// ---------------------------------------------------------------------------
template <int kD, bool kBF16, int kStages>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr,
                                         uint32_t issue) {
  using L = FwdLayout<kD, kBF16, kStages>;
  constexpr uint32_t kIdesc = idesc_f16_f32(128, 128, kBF16, false);
  const uint32_t q_lo = sdesc_lo(q_addr, 16), k_lo = sdesc_lo(k_addr, 16);
#pragma unroll
  for (int k = 0; k < kD / 16; ++k) {
    // K-major SW128: 16-element (32-byte) steps inside a 64-element atom,
    // then the next atom (next TMA box) for head_dim >= 64.
    const uint32_t off = (k / 4) * L::kAtomBytes + (k % 4) * 32u;
    // The 14-bit address field of the base descriptor plus the step in 16-byte
    // units: shared-memory addresses stay below 2^18 bytes, so nothing carries
    // out of the field and the result equals sdesc_lo(addr + off) -- one add
    // per operand instead of a full descriptor computation per K step (fewer
    // instructions on the MMA warp's sub-partition, which it shares with two
    // softmax warps).
    umma_f16_ss(d_tmem, q_lo + (off >> 4), k_lo + (off >> 4), kIdesc, k > 0 ? 1u : 0u, issue);
  }
}

// O (+)= P[:, chunk] V[chunk, :] for one P chunk (kPvStepsPerChunk K-steps).
template <int kD, bool kBF16, int kStages>
__device__ __forceinline__ void issue_pv_chunk(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_addr,
                                               int chunk, bool accumulate, uint32_t issue) {
  using L = FwdLayout<kD, kBF16, kStages>;
  constexpr uint32_t kIdesc = idesc_f16_f32(128, kD, kBF16, true);
  const uint32_t v_lo = sdesc_lo(v_addr, L::kAtomBytes);
#pragma unroll
  for (int k = L::chunk_begin(chunk) / 16; k < L::chunk_begin(chunk + 1) / 16; ++k) {
    const int i = k - L::chunk_begin(chunk) / 16;
    // V is MN-major (head_dim contiguous): 8-row groups 1024 B apart (SBO),
    // 64-element head_dim atoms one TMA box apart (LBO); 16 key rows per step.
    // P in TMEM: 16 elements of 16 bit = 8 columns per K step.
    umma_f16_ts(d_tmem, p_tmem + k * 8u, v_lo + static_cast<uint32_t>(k) * (16u * 128u >> 4), kIdesc,
                (accumulate || i > 0) ? 1u : 0u, issue);
  }
}

template <int kD, bool kBF16, int kStages, bool kCausal>
__device__ __forceinline__ void role_mma(const FwdParams& p, uint32_t sbase, uint32_t bar0,
                                         uint32_t tmem, const CtaSync& sy, const WorkQueue<4>& wq) {
  using L = FwdLayout<kD, kBF16, kStages>;
  auto bar = [&](int i) { return bar0 + 8u * static_cast<uint32_t>(i); };
  auto slot_addr = [&](uint32_t s) { return sbase + L::kOffKV + s * L::kTileBytes; };
  const uint32_t tS[2] = {tmem + 0u, tmem + 128u};
  const uint32_t tO[2] = {tmem + L::kColO, tmem + L::kColO + kD};
  const uint32_t qa[2] = {sbase + L::kOffQ, sbase + L::kOffQ + L::kTileBytes};
  // The whole warp runs this role in converged control flow; lane 0 issues.
  const uint32_t leader = (threadIdx.x & 31u) == 0u ? 1u : 0u;
  uint32_t kv_cnt = 0, it = 0;
  uint32_t pph[2] = {0u, 0u};
  // O_wg (+)= P_wg V: each P chunk is issued as soon as its barrier flips.
  auto pv = [&](int wg, uint32_t v_addr, bool accumulate) -> bool {
    if constexpr (L::kCorr) {
      // The first PV of an item overwrites O_wg: the correction warps must
      // have read out the previous item's O_wg.
      if (!accumulate && it > 0u && !sy.wait(bar(L::kBarOFree + wg), (it - 1u) & 1u, kSiteMmaOFree))
        return false;
    }
#pragma unroll
    for (int c = 0; c < L::kPChunks; ++c) {
      if (!sy.wait(bar(L::kBarPReady + wg * L::kPChunks + c), pph[wg], wg ? kSiteMmaP1 : kSiteMmaP0))
        return false;
      tc_fence_after_sync();
      issue_pv_chunk<kD, kBF16, kStages>(tO[wg], tS[wg], v_addr, c, accumulate || c > 0, leader);
    }
    pph[wg] ^= 1u;
    return true;
  };
  bool ok = (p.test_flags & 2u) == 0u;  // bit 1: issue nothing; the other roles' waits run out
  // The next work item's first S0 is issued before the current item's last
  // PV1 (after its last PV0), so Q tile 0's warpgroup finds it ready after
  // its epilogue instead of after Q tile 1's last softmax and PV (the item
  // boundary of short sequences).  Its K_0 can load by then: of the ring only
  // the last V is still held.  Not in the causal kernel at head_dim 128,
  // where it measured 0.3-1.3 % slower (+0.8-3.3 % at head_dim 64).
#ifndef AFA_EAGER_S0
#define AFA_EAGER_S0 1
#endif
#ifndef AFA_EAGER_S0_CAUSAL_D128
#define AFA_EAGER_S0_CAUSAL_D128 0
#endif
  constexpr bool kEagerS0 =
      AFA_EAGER_S0 != 0 && (!kCausal || kD == 64 || AFA_EAGER_S0_CAUSAL_D128 != 0);
  bool s0_early = false;   // this item's S0(0) was issued during the previous item
  bool have_next = false;  // the next item was read from the queue already
  int w_next = 0;
  for (; ok; ++it) {
    const int w = have_next ? w_next : wq.next(it, sy, kSiteReadItem);
    have_next = false;
    if (w < 0) break;  // done, or aborted
    // Q tile 0 visits n0 K/V tiles, Q tile 1 n1 >= n0 (equal without a causal
    // mask; the work item is only decoded when they can differ).
    int n0 = p.n_kv, n1 = p.n_kv;
    if (kCausal) {
      int qp, h, b;
      decode_work<kCausal>(p, w, qp, h, b);
      n0 = kv_tiles<kCausal>(p, qp, 0);
      n1 = kv_tiles<kCausal>(p, qp, 1);
    }
    uint32_t ks = kv_cnt % kStages;
    if (!s0_early) {
      if (!sy.wait(bar(L::kBarQFull + 0), it & 1u, kSiteMmaQFull)) { ok = false; break; }
      if (!sy.wait(bar(L::kBarKVFull + ks), (kv_cnt / kStages) & 1u, kSiteMmaKFull)) { ok = false; break; }
      tc_fence_after_sync();
      issue_qk<kD, kBF16, kStages>(tS[0], qa[0], slot_addr(ks), leader);
      umma_commit(bar(L::kBarSFull + 0), leader);
      if (n0 == 1) umma_commit(bar(L::kBarQEmpty + 0), leader);  // last S0 of the item issued
    }
    s0_early = false;
    if (!sy.wait(bar(L::kBarQFull + 1), it & 1u, kSiteMmaQFull)) { ok = false; break; }
    tc_fence_after_sync();
    issue_qk<kD, kBF16, kStages>(tS[1], qa[1], slot_addr(ks), leader);
    umma_commit(bar(L::kBarSFull + 1), leader);
    umma_commit(bar(L::kBarKVEmpty + ks), leader);
    ++kv_cnt;
    uint32_t vcnt = kv_cnt++;
    for (int j = 1; j < n1; ++j) {
      ks = kv_cnt % kStages;
      const uint32_t vs = vcnt % kStages;
      if (!sy.wait(bar(L::kBarKVFull + vs), (vcnt / kStages) & 1u, kSiteMmaVFull)) { ok = false; break; }
      if (!sy.wait(bar(L::kBarKVFull + ks), (kv_cnt / kStages) & 1u, kSiteMmaKFull)) { ok = false; break; }
      // Tensor-core order PV0(j-1), S0(j), PV1(j-1), S1(j): S_i(j) overwrites
      // the TMEM columns P_i(j-1) was read from, after that PV in issue order.
      // Q tile 0 stops after n0 tiles (causal): its last PV completes O0.
      if (j - 1 < n0) {
        if (!pv(0, slot_addr(vs), j > 1)) { ok = false; break; }
        if (j == n0) umma_commit(bar(L::kBarOFinal + 0), leader);
      }
      if (j < n0) {
        issue_qk<kD, kBF16, kStages>(tS[0], qa[0], slot_addr(ks), leader);
        umma_commit(bar(L::kBarSFull + 0), leader);
        if (j == n0 - 1) umma_commit(bar(L::kBarQEmpty + 0), leader);  // last S0 of the item
      }
      if (!pv(1, slot_addr(vs), j > 1)) { ok = false; break; }
      umma_commit(bar(L::kBarKVEmpty + vs), leader);
      issue_qk<kD, kBF16, kStages>(tS[1], qa[1], slot_addr(ks), leader);
      umma_commit(bar(L::kBarSFull + 1), leader);
      umma_commit(bar(L::kBarKVEmpty + ks), leader);
      ++kv_cnt;
      vcnt = kv_cnt++;
    }
    if (!ok) break;
    umma_commit(bar(L::kBarQEmpty + 1), leader);  // last S1 of the item issued: Q1 may be reloaded
    const uint32_t vs = vcnt % kStages;
    if (!sy.wait(bar(L::kBarKVFull + vs), (vcnt / kStages) & 1u, kSiteMmaVFull)) { ok = false; break; }
    if (n0 == n1) {
      if (!pv(0, slot_addr(vs), n1 > 1)) { ok = false; break; }
      umma_commit(bar(L::kBarOFinal + 0), leader);
    }
    if constexpr (kEagerS0) {
      // The next item (read once; the next iteration takes it from here) and
      // its K_0, whose ring slot is not the one V is in.
      w_next = wq.next(it + 1u, sy, kSiteReadItem);
      have_next = true;
      if (w_next >= 0) {
        int n0n = p.n_kv;
        if (kCausal) {
          int qp, h, b;
          decode_work<kCausal>(p, w_next, qp, h, b);
          n0n = kv_tiles<kCausal>(p, qp, 0);
        }
        const uint32_t kn = kv_cnt % kStages;
        if (!sy.wait(bar(L::kBarQFull + 0), (it + 1u) & 1u, kSiteMmaQFull)) { ok = false; break; }
        if (!sy.wait(bar(L::kBarKVFull + kn), (kv_cnt / kStages) & 1u, kSiteMmaKFull)) { ok = false; break; }
        tc_fence_after_sync();
        issue_qk<kD, kBF16, kStages>(tS[0], qa[0], slot_addr(kn), leader);
        umma_commit(bar(L::kBarSFull + 0), leader);
        if (n0n == 1) umma_commit(bar(L::kBarQEmpty + 0), leader);
        s0_early = true;
      }
    }
    if (!pv(1, slot_addr(vs), n1 > 1)) { ok = false; break; }
    umma_commit(bar(L::kBarOFinal + 1), leader);
    umma_commit(bar(L::kBarKVEmpty + vs), leader);
  }
  // Drain: every MMA issued by this thread has completed before teardown
  // releases tensor memory.
  umma_commit(bar(L::kBarMmaDrain), leader);
  if (!mbar_try_wait(bar(L::kBarMmaDrain), 0)) sy.wait_slow(bar(L::kBarMmaDrain), 0, kSiteMmaDrain, false);
}

// ---------------------------------------------------------------------------
// Role: softmax + correction + epilogue (one warpgroup per Q tile)
// ---------------------------------------------------------------------------
template <int kD, bool kBF16, int kStages, bool kCausal>
__device__ __forceinline__ void role_softmax(const FwdParams& p, int wg, uint8_t* smem, uint32_t bar0,
                                             uint32_t tmem, const CtaSync& sy, const WorkQueue<4>& wq) {
  using L = FwdLayout<kD, kBF16, kStages>;
  using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  auto bar = [&](int i) { return bar0 + 8u * static_cast<uint32_t>(i); };
  const int warp_in_wg = (threadIdx.x >> 5) & 3;
  const int row = warp_in_wg * 32 + static_cast<int>(threadIdx.x & 31);
  const uint32_t lane_field = static_cast<uint32_t>(warp_in_wg * 32) << 16;
  const uint32_t tS = tmem + lane_field + static_cast<uint32_t>(wg) * 128u;
  const uint32_t tO = tmem + lane_field + L::kColO + static_cast<uint32_t>(wg) * kD;
  const float sl2 = p.scale_log2;
  const uint32_t bar_s = bar(L::kBarSFull + wg);
  const uint32_t bar_p0 = bar(L::kBarPReady + wg * L::kPChunks);
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t bar_o = bar(L::kBarOFinal + wg);
  uint32_t sph = 0, oph = 0;

  for (uint32_t it = 0;; ++it) {
    const int w = wq.next(it, sy, kSiteReadItem);
    if (w < 0) return;  // done, or aborted
    // The item's coordinates (integer divisions): needed up front only under
    // the causal mask; otherwise decoded while the final O is awaited, off
    // the item boundary.
    int qp = 0, h = 0, b = 0;
    if constexpr (kCausal) decode_work<kCausal>(p, w, qp, h, b);
    const int n_tiles = kv_tiles<kCausal>(p, qp, wg);
    // Keys this row sees: all seq_len_kv, or under the causal mask those with
    // index <= q_row + causal_off.
    const int row_keys =
        kCausal ? min(qp * 256 + wg * 128 + row + p.causal_off + 1, p.seq_len_kv) : p.seq_len_kv;
    float m_ref = -INFINITY;  // running reference max, already in log2 units (x scale*log2e)
    float l = 0.f;
    for (int j = 0; j < n_tiles; ++j) {
      if (!sy.wait(bar_s, sph, kSiteSoftmaxS)) return;
      sph ^= 1u;
      tc_fence_after_sync();
      uint32_t sr[128];
      tmem_ld64_sync(tS, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
      tmem_ld64_sync(tS + 64u, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
      float s[128];
#pragma unroll
      for (int k = 0; k < 128; ++k) s[k] = __uint_as_float(sr[k]);
      const int valid = row_keys - j * 128;  // key columns of this tile this row sees
      // Without the causal mask `valid` is the same for every row of the tile.
      if (kCausal ? __any_sync(0xffffffffu, valid < 128) : valid < 128) {
#pragma unroll
        for (int k = 0; k < 128; ++k) s[k] = (k < valid) ? s[k] : -INFINITY;
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int k = 0; k < 128; k += 8) {
        mx0 = fmax3(mx0, s[k], s[k + 1]);
        mx1 = fmax3(mx1, s[k + 2], s[k + 3]);
        mx2 = fmax3(mx2, s[k + 4], s[k + 5]);
        mx3 = fmax3(mx3, s[k + 6], s[k + 7]);
      }
      const float m_new = fmaxf(fmax3(mx0, mx1, mx2), mx3) * sl2;
      const bool need = m_new > m_ref + 8.0f;
      // alpha rescales the running sum and O from the old reference max.
      const float alpha = need ? ex2_approx(m_ref - m_new) : 1.0f;
      if constexpr (L::kCorr) {
        // The correction warp of this quadrant rescales O (if any row of the
        // warp needs it) and then releases P chunk 0 together with this warp.
        // It gets the reference maximum before and after this tile and forms
        // the factor itself, so no exponential precedes the hand-over here.
        if (j > 0) {
          reinterpret_cast<float2*>(smem + L::kOffAlpha)[wg * 128 + row] =
              make_float2(m_ref, need ? m_new : m_ref);
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(L::kBarAlpha + wg * 4 + warp_in_wg));
        }
      } else if (j > 0 && __any_sync(0xffffffffu, need)) {
        // Conditional rescale of O, before this step's first P chunk is handed
        // over: the previous PV of this tile has completed (it was committed
        // before S(j)) and the next one waits for that chunk, so O is quiescent.
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32_sync(tO + c * 32u, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + c * 32u, o);
        }
      }
      if (need) m_ref = m_new;
      const float2 c2 = make_float2(sl2, sl2);
      // A row that has seen no key yet (causal mask) keeps m_ref = -inf; its
      // masked scores then give exp2(-inf) = 0 instead of exp2(-inf + inf).
      const float m_use = (kCausal && m_ref == -INFINITY) ? 0.f : m_ref;
      const float2 nm2 = make_float2(-m_use, -m_use);
      float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
      uint32_t pk[64];
      // P = exp2(S * scale*log2e - m_ref) for one chunk of kSColsPerChunk columns.
      auto exp_chunk = [&](int c) {
#pragma unroll
        for (int k = L::chunk_begin(c); k < L::chunk_begin(c + 1); k += 2) {
          const float2 x = __ffma2_rn(make_float2(s[k], s[k + 1]), c2, nm2);
          float2 e;
          if ((((k >> 1) * L::kEmuPairs) & 7) < L::kEmuPairs) {
            e = exp2_fma_pipe2(x);
          } else {
            e.x = ex2_approx(x.x);
            e.y = ex2_approx(x.y);
          }
          if ((k >> 1) & 1)
            acc1 = __fadd2_rn(acc1, e);
          else
            acc0 = __fadd2_rn(acc0, e);
          pk[k >> 1] = pack2<kBF16>(e.x, e.y);
        }
      };
      // Chunk c's P is in TMEM (and any O rescale done): release it to the MMA.
      auto hand_off = [&](int c) {
        tmem_wait_st();
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          // With the correction warpgroup, chunk 0 also counts the correction
          // warp of this quadrant, which has nothing to do on a first tile.
          if (L::kCorr && c == 0 && j == 0)
            mbar_arrive_cnt(bar_p0, 2u);
          else
            mbar_arrive(bar_p0 + 8u * static_cast<uint32_t>(c));
        }
      };
      // Software-pipelined by one chunk: the store of chunk c-1 drains while
      // chunk c is computed.
      auto store_chunk = [&](int c) {
#pragma unroll
        for (int q = L::chunk_begin(c) / 2; q < L::chunk_begin(c + 1) / 2; q += 16)
          tmem_st16(tS + q, &pk[q]);
      };
      exp_chunk(0);
      store_chunk(0);
#pragma unroll
      for (int c = 1; c < L::kPChunks; ++c) {
        exp_chunk(c);
        hand_off(c - 1);
        store_chunk(c);
      }
      hand_off(L::kPChunks - 1);
      l = l * alpha + ((acc0.x + acc1.x) + (acc0.y + acc1.y));
    }
    if constexpr (L::kCorr) {
      // The correction warpgroup runs the epilogue from these row statistics
      // (two slots: this warp may finish the next item before they are read).
      // (Plain stores and loads: the mbarrier arrive / wait around them are
      // compiler memory barriers with release / acquire semantics.)
      reinterpret_cast<float2*>(smem + L::kOffStats)[((it & 1u) * 2u + wg) * 128u + row] = make_float2(l, m_ref);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::kBarStats + wg * 4 + warp_in_wg));
      continue;
    }
    // Epilogue: O / l, round to the input type, store the row.  A row that
    // saw no key (causal mask) has l = 0 and O = 0: it stores 0, and a
    // log-sum-exp of -inf.
    if constexpr (!kCausal) decode_work<kCausal>(p, w, qp, h, b);
    const int q_row = qp * 256 + wg * 128 + row;
    if (!sy.wait(bar_o, oph, kSiteSoftmaxO)) return;
    oph ^= 1u;
    tc_fence_after_sync();
    const float inv_l = l > 0.f ? 1.0f / l : 0.f;
    const bool row_ok = q_row < p.seq_len;
    if (p.lse != nullptr && row_ok) {
      // ln(sum_j exp(s_j * scale)) = (m_ref + log2(l)) * ln(2), m_ref in log2 units.
      const float lse = l > 0.f ? (m_ref + log2f(l)) * 0.69314718055994531f : -INFINITY;
      p.lse[(static_cast<long long>(b) * p.n_heads + h) * p.seq_len + q_row] = lse;
    }
    if constexpr (L::kOTma) {
      // 64-column pieces of this warp's 32 rows go to its staging tile (16-byte
      // chunk k of a row at chunk position k ^ (row % 8), the 128-byte swizzle
      // of the O tensor map) and out with one TMA store each; rows past
      // seq_len are clipped by the store.
      const uint32_t stage = smem_u32(smem) + L::kOffStage +
                             static_cast<uint32_t>(wg * 4 + warp_in_wg) * L::kStageBytes;
      const int row0 = qp * 256 + wg * 128 + warp_in_wg * 32;
      const bool si = (p.seq_inner_mask & 8u) != 0u;
      // Piece c + 1 is read from TMEM and rounded while piece c's store is
      // still reading the staging tile.
      uint32_t pc[32];
      auto load_piece = [&](int c) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t o[32];
          tmem_ld32_sync(tO + static_cast<uint32_t>(c * 64 + hh * 32), o);
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pc[hh * 16 + e] = pack2<kBF16>(__uint_as_float(o[2 * e]) * inv_l, __uint_as_float(o[2 * e + 1]) * inv_l);
        }
      };
      load_piece(0);
#pragma unroll
      for (int c = 0; c < kD / 64; ++c) {
        if (lane == 0) bulk_wait_group_read<0>();  // the previous store has read the tile
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          st_shared_v4(stage + lane * 128u + ((static_cast<uint32_t>(k) ^ (lane & 7u)) << 4), pc[4 * k],
                       pc[4 * k + 1], pc[4 * k + 2], pc[4 * k + 3]);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0 && row0 < p.seq_len) {
          tma_store_4d(&p.tm_o, stage, c * 64, si ? row0 : h, si ? h : row0, b);
          bulk_commit_group();
        }
        if (c + 1 < kD / 64) load_piece(c + 1);
      }
      tc_fence_before_sync();
      continue;
    }
    T* orow = static_cast<T*>(p.o) + static_cast<long long>(b) * p.o_sb +
              static_cast<long long>(q_row) * p.o_sn + static_cast<long long>(h) * p.o_sh;
#pragma unroll
    for (int c = 0; c < kD / 32; ++c) {
      uint32_t o[32];
      tmem_ld32_sync(tO + c * 32u, o);
      uint32_t pk[16];
#pragma unroll
      for (int e = 0; e < 16; ++e)
        pk[e] = pack2<kBF16>(__uint_as_float(o[2 * e]) * inv_l, __uint_as_float(o[2 * e + 1]) * inv_l);
      if (row_ok) {
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4)
          st_global_v4(orow + c * 32 + v4 * 8, pk[4 * v4], pk[4 * v4 + 1], pk[4 * v4 + 2],
                       pk[4 * v4 + 3]);
      }
    }
    tc_fence_before_sync();
  }
}

// ---------------------------------------------------------------------------
// Role: correction + epilogue (fourth warpgroup, AFA_CORRECTION_WG only)
// ---------------------------------------------------------------------------
// Warp q of the warpgroup reaches TMEM lane quadrant q: rows 32q..32q+31 of
// both Q tiles.  Per K/V tile j > 0 of each Q tile it takes the row scale
// factors its softmax peer wrote, rescales those O rows in TMEM when any of
// them changed (the PV of tile j-1 has completed: the peer saw S(j), committed
// after it) and then arrives on P chunk 0's barrier, so PV(j) follows the
// rescale.  After an item's final PV it writes O * 1/l (and the log-sum-exp):
// 64-column pieces are rounded into a 128-byte-swizzled staging tile and
// written by TMA stores, and O is released to the next item's first PV as
// soon as it has been read from TMEM.  Events are taken in a fixed order --
// the tiles' scale factors, then the epilogues of Q tile 0 and 1 -- which the
// MMA issue order makes deadlock-free.
// Numerics as the reference: rescale by exp2(m_old - m_new)
// (csrc/include/afa_softmax.cuh:50-68), final O / l (:109-127).
template <int kD, bool kBF16, int kStages, bool kCausal>
__device__ __forceinline__ void role_correction(const FwdParams& p, uint8_t* smem, uint32_t sbase,
                                                uint32_t bar0, uint32_t tmem, const CtaSync& sy,
                                                const WorkQueue<4>& wq) {
  using L = FwdLayout<kD, kBF16, kStages>;
  auto bar = [&](int i) { return bar0 + 8u * static_cast<uint32_t>(i); };
  const int quad = static_cast<int>((threadIdx.x >> 5) & 3u);
  const uint32_t lane = threadIdx.x & 31u;
  const int row = quad * 32 + static_cast<int>(lane);
  const uint32_t lane_field = static_cast<uint32_t>(quad * 32) << 16;
  const float2* alpha_s = reinterpret_cast<const float2*>(smem + L::kOffAlpha);
  const float2* stats_s = reinterpret_cast<const float2*>(smem + L::kOffStats);
  const uint32_t stage = sbase + L::kOffStage + static_cast<uint32_t>(quad) * L::kStageBytes;
  const bool si = (p.seq_inner_mask & 8u) != 0u;
  // Barrier phases, bit wg for Q tile wg (bit masks, not arrays: indexed by a
  // loop variable an array would live in local memory).
  uint32_t aph = 0u, sph = 0u, oph = 0u;
  bool ok = true;
  for (uint32_t it = 0; ok; ++it) {
    const int w = wq.next(it, sy, kSiteReadItem);
    if (w < 0) break;
    int qp, h, b;
    decode_work<kCausal>(p, w, qp, h, b);
    const int n0 = kv_tiles<kCausal>(p, qp, 0), n1 = kv_tiles<kCausal>(p, qp, 1);
    for (int j = 1; j < n1 && ok; ++j) {
#pragma unroll
      for (int wg = 0; wg < 2; ++wg) {
        if (wg == 0 && j >= n0) continue;
        if (!sy.wait(bar(L::kBarAlpha + wg * 4 + quad), (aph >> wg) & 1u, kSiteCorrAlpha)) { ok = false; break; }
        aph ^= 1u << wg;
        // The softmax warp's factor exp2(m_old - m_new) when its reference
        // maximum moved, else 1 (the same instruction on the same operands).
        const float2 mm = alpha_s[wg * 128 + row];
        const bool moved = mm.y != mm.x;
        if (__any_sync(0xffffffffu, moved)) {
          const float a = moved ? ex2_approx(mm.x - mm.y) : 1.0f;
          tc_fence_after_sync();
          const uint32_t tO = tmem + lane_field + L::kColO + static_cast<uint32_t>(wg * kD);
#pragma unroll 1
          for (int c = 0; c < kD / 8; ++c) {
            uint32_t o[8];
            tmem_ld8_sync(tO + c * 8u, o);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * a);
            tmem_st8(tO + c * 8u, o);
          }
          tmem_wait_st();
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(L::kBarPReady + wg * L::kPChunks));
      }
    }
    if (!ok) break;
#pragma unroll 1
    for (int wg = 0; wg < 2; ++wg) {
      if (!sy.wait(bar(L::kBarStats + wg * 4 + quad), (sph >> wg) & 1u, kSiteCorrStats)) { ok = false; break; }
      sph ^= 1u << wg;
      if (!sy.wait(bar(L::kBarOFinal + wg), (oph >> wg) & 1u, kSiteSoftmaxO)) { ok = false; break; }
      oph ^= 1u << wg;
      tc_fence_after_sync();
      const float2 st = stats_s[((it & 1u) * 2u + wg) * 128u + row];
      const float l = st.x, m_ref = st.y;
      const int row0 = qp * 256 + wg * 128 + quad * 32;
      const int q_row = row0 + static_cast<int>(lane);
      if (p.lse != nullptr && q_row < p.seq_len) {
        // ln(sum_j exp(s_j * scale)) = (m_ref + log2(l)) * ln(2), m_ref in log2 units.
        const float lse = l > 0.f ? (m_ref + log2f(l)) * 0.69314718055994531f : -INFINITY;
        p.lse[(static_cast<long long>(b) * p.n_heads + h) * p.seq_len + q_row] = lse;
      }
      const float inv_l = l > 0.f ? 1.0f / l : 0.f;
      const uint32_t tO = tmem + lane_field + L::kColO + static_cast<uint32_t>(wg * kD);
#pragma unroll 1
      for (int c = 0; c < kD / 64; ++c) {
        // The staging tile is free once the previous store has read it.
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
#pragma unroll 1
        for (uint32_t k = 0; k < 8u; ++k) {  // 8 columns = one 16-byte chunk of the row
          uint32_t o[8];
          tmem_ld8_sync(tO + static_cast<uint32_t>(c * 64) + k * 8u, o);
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pk[e] = pack2<kBF16>(__uint_as_float(o[2 * e]) * inv_l, __uint_as_float(o[2 * e + 1]) * inv_l);
          // 16-byte chunk k of this row goes to chunk position k ^ (row % 8).
          st_shared_v4(stage + lane * 128u + ((k ^ (lane & 7u)) << 4), pk[0], pk[1], pk[2], pk[3]);
        }
        if (c == kD / 64 - 1) {
          // All of O_wg's rows of this warp have been read: the next item's
          // first PV may overwrite them.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(L::kBarOFree + wg));
        }
        fence_proxy_async_shared();
        __syncwarp();
        // Rows past seq_len are clipped by the store; a tile wholly past it is skipped.
        if (lane == 0 && row0 < p.seq_len) {
          tma_store_4d(&p.tm_o, stage, c * 64, si ? row0 : h, si ? h : row0, b);
          bulk_commit_group();
        }
      }
    }
  }
  // Every store has finished before the CTA (and its shared memory) goes away.
  if (lane == 0) bulk_wait_group<0>();
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------
template <int kD, bool kBF16, int kStages, bool kCausal>
__global__ void __launch_bounds__(FwdLayout<kD, kBF16, kStages>::kThreads, 1)
    afa_fwd_sm100_kernel(const __grid_constant__ FwdParams p) {
  using L = FwdLayout<kD, kBF16, kStages>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  const uint32_t bar0 = sbase + L::kOffBar;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const uint32_t lane = threadIdx.x & 31u;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < L::kNumBars; ++i) {
      // p_ready: one elected arrival per softmax warp; all others: one arrival.
      uint32_t count = 1u;
      if (i >= L::kBarPReady && i < L::kBarPReady + 2 * L::kPChunks)
        count = (L::kCorr && (i - L::kBarPReady) % L::kPChunks == 0) ? 8u : 4u;
      if (L::kCorr && i >= L::kBarOFree && i < L::kBarOFree + 2) count = 4u;
      if (i >= L::kBarItemEmpty && i < L::kBarItemEmpty + L::kItemSlots) count = L::kItemReaders;
      mbar_init(bar0 + 8u * i, count);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    if (L::kCorr || L::kOTma) tma_prefetch_desc(&p.tm_o);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const CtaSync sy{abort_flag, p.status, p.timeout_ns};
  // Dynamic schedule only for the causal kernel (items of unequal length) and
  // only with caller-provided scheduler words.
  const WorkQueue<L::kItemSlots> wq{kCausal ? p.sched : nullptr,
                                    reinterpret_cast<volatile int*>(smem + L::kOffItems),
                                    bar0 + 8u * L::kBarItemFull, bar0 + 8u * L::kBarItemEmpty, p.n_work,
                                    (p.test_flags & 4u) != 0u};

  if (warp < 4) {
    setmaxnreg_dec<L::kProducerRegs>();
    if (warp == 0) {
      role_load<kD, kBF16, kStages, kCausal>(p, sbase, bar0, sy, wq);
    } else if (warp == 1) {
      role_mma<kD, kBF16, kStages, kCausal>(p, sbase, bar0, tmem, sy, wq);
    }
  } else if (warp < 12) {
    setmaxnreg_inc<L::kSoftmaxRegs>();
    role_softmax<kD, kBF16, kStages, kCausal>(p, (warp - 4) >> 2, smem, bar0, tmem, sy, wq);
    // Every TMA store of O has finished before the CTA (and its shared memory) goes away.
    if (L::kOTma && lane == 0) bulk_wait_group<0>();
  } else {
    if constexpr (L::kCorr) {
      setmaxnreg_dec<L::kCorrRegs>();
      role_correction<kD, kBF16, kStages, kCausal>(p, smem, sbase, bar0, tmem, sy, wq);
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace afa100
