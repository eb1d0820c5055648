/*
 * afa_sm100.h -- C ABI of the B200 (sm_100a) attention-forward library
 * (libafa_sm100.so).
 *
 * Computes the attention forward  O = softmax(Q K^T * scale) V  for fp16/bf16
 * tensors laid out as [batch, seq_len, n_heads, head_dim].  With the extension
 * fields of AfaFwdArgs left zero it is exactly the operation and layout of the
 * reference's torch binding `afa_flash_attention_kernels.forward`
 * (csrc/ampere_flash_attention.cu:35-136): non-causal, K and V shaped like Q.
 * The extensions add a K/V length different from the query length, grouped
 * K/V heads (GQA), a causal mask and a log-sum-exp output.
 *
 * Plain C types only: pointers are device addresses, the stream is a
 * cudaStream_t passed as void*.  No call allocates, frees or synchronizes; all
 * buffers belong to the caller.  Every entry point returns an AFA_* status code
 * and never throws.
 */
#ifndef AFA_SM100_H_
#define AFA_SM100_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types: the integer values of torch's ScalarType, as used by the
 * reference's Python DType enum (afa_py/afa_config.py:8-28: FP16 = 5, BF16 = 15). */
#define AFA_DTYPE_FP16 5
#define AFA_DTYPE_BF16 15

/* Return codes. */
#define AFA_OK 0
#define AFA_ERR_INVALID_ARGUMENT 1   /* null pointer, non-positive size, n_kv_heads not dividing n_heads, causal not 0/1 */
#define AFA_ERR_UNSUPPORTED_DTYPE 2  /* dtype not fp16/bf16 */
#define AFA_ERR_NO_KERNEL 3          /* no compiled kernel for (dtype, head_dim) */
#define AFA_ERR_MISALIGNED 4         /* base address / stride not 16-byte aligned (lse: 4, sched: 8) */
#define AFA_ERR_NO_DEVICE 5          /* no current CUDA device */
#define AFA_ERR_ARCH 6               /* device is not compute capability 10.0 */
#define AFA_ERR_TENSOR_MAP 7         /* cuTensorMapEncodeTiled rejected a tensor */
#define AFA_ERR_LAUNCH 8             /* kernel launch failed */
#define AFA_ERR_DEVICE_TIMEOUT 9     /* a device-side bounded wait ran out (status word) */
#define AFA_ERR_TOO_LARGE 10         /* a size exceeds what the kernel indexes */
#define AFA_ERR_SCRATCH_LIMIT 11     /* afa_fwd_sm100_noalloc: the call needs more scratch than
                                        AFA_NOALLOC_SCRATCH_BYTES */

/* Arguments of one forward call.  Strides are in elements, for the
 * (batch, seq, head) dimensions; head_dim must be contiguous (stride 1).
 * Q and O are [batch, seq_len, n_heads, head_dim]; K and V are
 * [batch, seq_len_kv, n_kv_heads, head_dim].
 * Replaces the reference's AFAForwardParams (csrc/include/afa_config.cuh:7-34),
 * which had one stride set shared by all four tensors and one shape. */
typedef struct AfaFwdArgs {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t q_strides[3];
  int64_t k_strides[3];
  int64_t v_strides[3];
  int64_t o_strides[3];
  int32_t batch;
  int32_t seq_len;
  int32_t n_heads;
  int32_t head_dim;   /* 64 or 128 */
  int32_t dtype;      /* AFA_DTYPE_FP16 or AFA_DTYPE_BF16 */
  float scale;        /* softmax scale; <= 0 selects 1/sqrt(head_dim) as the reference */
  int32_t* status;    /* optional int32 the kernel can address -- device memory, or mapped
                          page-locked host memory (cudaHostAllocMapped) so the host can read
                          it without synchronising: 0 = ok, else an AFA_DEV_* code (see below) */
  uint64_t timeout_ns; /* bound of every device-side wait; 0 selects the default (4 s) */
  uint32_t test_flags; /* 0 in normal use; AFA_TEST_* bits below exercise failure paths */
  /* Extensions (ABI 2.0: seq_len_kv, n_kv_heads, causal, lse; 3.0: sched); zero everywhere gives
     the reference's operation. */
  int32_t seq_len_kv;  /* rows of K and V; 0 selects seq_len */
  int32_t n_kv_heads;  /* heads of K and V, a divisor of n_heads (query head h reads
                          K/V head h / (n_heads / n_kv_heads)); 0 selects n_heads */
  int32_t causal;      /* 1: query row i sees only keys j <= i + seq_len_kv - seq_len
                          (bottom-right aligned, the FlashAttention convention); a row
                          that sees no key gets O = 0.  0: no mask */
  float* lse;          /* optional device fp32 [batch, n_heads, seq_len], contiguous:
                          ln(sum_j exp(scale * q_i . k_j)) over the keys row i sees,
                          -inf for a row that sees none.  NULL: not written */
  int32_t* sched;      /* optional device int32[2], 8-byte aligned, zero before first use:
                          scheduler words of the causal kernel, which then hands out work
                          items dynamically (atomic counter) instead of round-robin; the
                          kernel returns them to zero when it ends.  One launch at a time
                          per pair of words: launches that may overlap (other streams) need
                          their own.  Ignored without the causal mask.  NULL: static schedule */
} AfaFwdArgs;

/* test_flags bit: the kernel's TMA producer issues no loads, so the first
 * bounded wait of the MMA issuer runs out after timeout_ns.  The kernel then
 * writes AFA_DEV_TIMEOUT_BASE + site to the status word and returns; nothing is
 * in flight, the context stays usable.  Lets a test observe the device-side
 * timeout path without hanging or faulting a GPU. */
#define AFA_TEST_PRODUCER_IDLE 1u
/* test_flags bit: the MMA issuer issues nothing, so the producer fills the
 * K/V ring and its bounded wait for a free slot runs out while its loads have
 * landed or are landing: it waits (bounded) for them before the CTA exits, and
 * the softmax warps' waits for S run out too.  Status word and context as for
 * AFA_TEST_PRODUCER_IDLE. */
#define AFA_TEST_MMA_IDLE 2u
/* test_flags bit (causal kernel with scheduler words): the kernel runs normally
 * but does not return the scheduler words to zero when it ends, so a test can
 * check that the next call's words are cleared (afa_fwd_sm100_noalloc). */
#define AFA_TEST_KEEP_SCHED 4u

/*
 * Launch the forward kernel on `stream` (a cudaStream_t) for the current device.
 * Replaces the launch path of the reference's flash_attention_forward
 * (csrc/ampere_flash_attention.cu:35-136) and its kernel table lookup
 * (csrc/include/afa_preset_kernels.cuh:10-54), keyed here on (dtype, head_dim).
 * Asynchronous: returns after the launch.  Argument errors are reported before
 * any CUDA call is made.
 */
int afa_fwd_sm100(const AfaFwdArgs* args, void* stream);

/*
 * afa_fwd_sm100 for callers that must not allocate device memory.  (No
 * counterpart in the reference, whose binding allocates through torch.)
 *
 * Who needs it: code that runs where cudaMalloc is off limits -- a plugin
 * inside a host framework that owns every device allocation and forbids
 * private ones, or a latency-critical path that cannot afford cudaMalloc's
 * implicit device-wide synchronisation -- and so cannot hand afa_fwd_sm100
 * the scheduler words (AfaFwdArgs.sched) the causal kernel uses as scratch.
 *
 * What it does instead: those words live in a static, 256-byte-aligned
 * __device__ array inside this library, AFA_NOALLOC_SCRATCH_BYTES (256 bytes)
 * per device, which every GPU that loads the library keeps until the process
 * exits.  The caller still passes inputs and outputs; args->sched must be NULL
 * (else AFA_ERR_INVALID_ARGUMENT), and a call that would need more scratch
 * than the array holds is refused with AFA_ERR_SCRATCH_LIMIT (today a call
 * needs at most 8 bytes).  Nothing is allocated or freed: before each causal
 * launch the entry point clears, with cudaMemsetAsync on `stream`, exactly the
 * words that must start at zero, because the array keeps whatever the previous
 * call left in it.
 *
 * Set-up: the first causal call on a device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current); make that first
 * call before any stream capture on the device.
 *
 * Races: every call on a device shares the array, so two causal calls whose
 * kernels may overlap on the GPU (different streams, or threads with no
 * ordering between them) corrupt each other's schedule; order them on one
 * stream, or give each its own words through afa_fwd_sm100.  Otherwise the
 * same as afa_fwd_sm100, with bit-identical results.
 */
#define AFA_NOALLOC_SCRATCH_BYTES 256
int afa_fwd_sm100_noalloc(const AfaFwdArgs* args, void* stream);

/* Human-readable text for an AFA_* return code (static storage). */
const char* afa_strerror(int code);

/*
 * Device status words written by the kernel into AfaFwdArgs.status (plain
 * stores: when several waits run out, the code of one of them remains; a
 * non-zero word is never overwritten by a later launch's code unless it is
 * first reset).  AFA_DEV_TIMEOUT_BASE + site: a bounded mbarrier wait at
 * `site` ran out and the kernel returned early (the output is then undefined).
 * Decodes a status word into text (static storage).
 */
#define AFA_DEV_OK 0
#define AFA_DEV_TIMEOUT_BASE 0x100
const char* afa_status_string(int32_t status);

/* 1 if a kernel is compiled for (dtype, head_dim), else 0.  Host-only. */
int afa_fwd_sm100_supported(int32_t dtype, int32_t head_dim);

/* Dynamic shared memory bytes and threads per CTA of the (dtype, head_dim)
 * kernel, or -1 if not compiled.  Host-only. */
int afa_fwd_sm100_smem_bytes(int32_t dtype, int32_t head_dim);
int afa_fwd_sm100_threads(void);

/* Library ABI version (major * 100 + minor). */
int afa_sm100_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* AFA_SM100_H_ */
