// afa_torch_binding.cpp -- the `afa_flash_attention_kernels` torch extension.
//
// Same Python surface as the reference binding
// (csrc/ampere_flash_attention.cu:138-151):
//     O, ms = afa_flash_attention_kernels.forward(kernel_cfg, q, k, v, o, benchmark=False)
// with the same checks and RuntimeError messages where the behaviour carries
// over (csrc/ampere_flash_attention.cu:39-99).  Underneath it calls the C ABI
// afa_fwd_sm100() (include/afa_sm100.h); this file holds no device code.
//
// Deliberate differences from the reference binding:
//   * the device must be compute capability 10.0 (the kernel is sm_100a code);
//   * the kernel table is keyed on (dtype, d_head) -- the Ampere tiling knobs
//     of the config are accepted and ignored;
//   * any seq_len >= 1 is accepted (no B_r/B_c divisibility rule) and inputs
//     may be strided views as long as head_dim is contiguous and the other
//     strides are multiples of 8 elements;
//   * `o` is checked against q's shape (the reference compared q with v);
//   * with benchmark=False the returned runtime is 0.0 (the reference returned
//     an uninitialised float); with benchmark=True the events are destroyed
//     and the launch's own status is checked after it finishes;
//   * every call first raises if an earlier launch on its device reported a
//     device-side abort (the reference checked nothing after its launch).
//
// One function beyond the reference:
//     O, lse = afa_flash_attention_kernels.forward_ext(q, k, v, o=None, causal=False,
//                                                      softmax_scale=None, return_lse=False)
// with K/V of their own length and head count (GQA), the causal mask and the
// fp32 log-sum-exp [batch, heads, seq] (None unless return_lse).
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CachingHostAllocator.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <optional>
#include <string>
#include <tuple>
#include <vector>

#include "afa_sm100.h"

namespace {

#define AFA_CHECK_CUDA(x) TORCH_CHECK((x).device().is_cuda(), #x " must be a CUDA tensor")
#define AFA_CHECK_LAST_DIM(x) \
  TORCH_CHECK((x).dim() == 4 && (x).stride(3) == 1, #x " must be 4-D [batch, seq, heads, head_dim] with a contiguous head_dim")

// The key fields of the Python AFAForwardKernelConfig.  All 13 attributes are
// read, as in py_to_cpp_kernel_config (csrc/ampere_flash_attention.cu:16-33),
// so a malformed config object fails the same way.
struct KernelKey {
  int dtype;
  int d_head;
};

KernelKey py_to_cpp_kernel_config(const py::object& cfg) {
  KernelKey key{py::cast<int>(cfg.attr("dtype")), py::cast<int>(cfg.attr("d_head"))};
  static const char* kInts[] = {"B_r", "B_c", "n_warps", "Q_col_fragments_per_warp_gemm",
                                "K_col_fragments_per_warp_gemm", "V_col_fragments_per_warp_gemm"};
  static const char* kBools[] = {"async_copy", "eager_load_blocks", "swizzled",
                                 "mma_double_buffer_loads", "optimized_softmax"};
  for (const char* a : kInts) (void)py::cast<int>(cfg.attr(a));
  for (const char* a : kBools) (void)py::cast<bool>(cfg.attr(a));
  return key;
}

int dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kHalf) return AFA_DTYPE_FP16;
  if (t.scalar_type() == at::kBFloat16) return AFA_DTYPE_BF16;
  return -1;
}

// One status word per device (int32, zero = ok) in mapped page-locked host
// memory: every launch on the device gets its device address, a kernel whose
// bounded wait runs out stores its code there, and the host reads it without
// synchronising.  Each call first takes (and clears) what earlier launches on
// its device reported, so a device-side abort is raised by the next call on
// that device -- at the latest by the first one made after the aborted launch
// has finished -- or by check_status(), which synchronises first.  Kept until
// the process exits (4 bytes of page-locked memory per device).
struct StatusWord {
  int32_t* host = nullptr;    // what the host reads
  int32_t* device = nullptr;  // the same word as the kernel addresses it
};
std::mutex g_status_mu;
std::map<int, StatusWord> g_status;

StatusWord status_word(int dev) {
  std::lock_guard<std::mutex> lock(g_status_mu);
  StatusWord& w = g_status[dev];
  if (w.host == nullptr) {
    void* h = nullptr;
    void* d = nullptr;
    TORCH_CHECK(cudaHostAlloc(&h, sizeof(int32_t), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess,
                "cudaHostAlloc of the status word failed");
    *static_cast<volatile int32_t*>(h) = 0;
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
      cudaFreeHost(h);
      TORCH_CHECK(false, "the device cannot address mapped host memory (status word)");
    }
    w.host = static_cast<int32_t*>(h);
    w.device = static_cast<int32_t*>(d);
  }
  return w;
}

// Takes the code earlier launches on `dev` left in the status word and clears it.
int32_t take_status(int dev) {
  return __atomic_exchange_n(status_word(dev).host, 0, __ATOMIC_ACQ_REL);
}

// Raises for an abort that a launch made before this call reported.
void raise_earlier_abort(int dev) {
  const int32_t st = take_status(dev);
  TORCH_CHECK(st == 0, "attention kernel reported (an earlier launch on cuda:", dev, "): ", afa_status_string(st));
}

// Scheduler words of the causal kernel (AfaFwdArgs.sched), one pair per
// (device, stream) so launches that may overlap never share them; zero at rest
// (the kernel returns them to zero when it ends, also after an abort).  A CUDA
// graph captured on a stream keeps that stream's pair: replays of it must be
// ordered with every other causal launch made on the capture stream, and two
// such graphs must not be replayed at the same time.
std::map<std::pair<int, cudaStream_t>, at::Tensor> g_sched;

int32_t* sched_words(const at::Device& dev, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_status_mu);
  at::Tensor& t = g_sched[{static_cast<int>(dev.index()), stream}];
  if (!t.defined()) t = at::zeros({2}, at::TensorOptions().dtype(at::kInt).device(dev));
  return t.data_ptr<int32_t>();
}

// Test hook: AFA_TEST_* flags and a wait bound for the next launch only
// (drives the kernel's bounded-wait abort through this binding).
std::mutex g_test_mu;
uint32_t g_test_flags = 0;
uint64_t g_test_timeout_ns = 0;

float launch(const at::Tensor& TQ, const at::Tensor& TK, const at::Tensor& TV, const at::Tensor& TO,
             int dt, float scale, bool causal, float* lse, bool benchmark);

std::tuple<at::Tensor, double> flash_attention_forward(const py::object& py_cfg,
                                                       const at::Tensor& TQ, const at::Tensor& TK,
                                                       const at::Tensor& TV,
                                                       std::optional<at::Tensor> out_,
                                                       bool benchmark) {
  AFA_CHECK_CUDA(TQ);
  AFA_CHECK_CUDA(TK);
  AFA_CHECK_CUDA(TV);
  AFA_CHECK_LAST_DIM(TQ);
  AFA_CHECK_LAST_DIM(TK);
  AFA_CHECK_LAST_DIM(TV);

  c10::cuda::CUDAGuard device_guard{TQ.device()};
  const int dev = TQ.device().index();
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  TORCH_CHECK(major == 10 && minor == 0,
              "Flash Attention (sm_100a build) requires SM_100 (current: SM_", major, ".", minor,
              ")");
  raise_earlier_abort(dev);

  const int dt = dtype_code(TQ);
  TORCH_CHECK(dt > 0, "Only fp16 and bf16 are supported");
  TORCH_CHECK(TK.dtype() == TQ.dtype(), "Input tensors must have the same data type");
  TORCH_CHECK(TV.dtype() == TQ.dtype(), "Input tensors must have the same data type");
  TORCH_CHECK(TK.device() == TQ.device() && TV.device() == TQ.device(),
              "Input tensors must be on the same device");

  const KernelKey cfg = py_to_cpp_kernel_config(py_cfg);
  TORCH_CHECK(afa_fwd_sm100_supported(cfg.dtype, cfg.d_head) == 1,
              "Kernel configuration was not found: no sm_100a kernel for dtype code ", cfg.dtype,
              ", d_head ", cfg.d_head);
  TORCH_CHECK(cfg.dtype == dt, "Kernel configuration dtype does not match input dtype");
  TORCH_CHECK(cfg.d_head == TQ.size(3), "Kernel configuration d_head (", cfg.d_head,
              ") does not match the input head_dim (", TQ.size(3), ")");

  TORCH_CHECK(TQ.sizes() == TK.sizes(), "Query and key tensors have same shape");
  TORCH_CHECK(TQ.sizes() == TV.sizes(), "Query and value tensors have same shape");
  TORCH_CHECK(TQ.size(0) > 0 && TQ.size(1) > 0 && TQ.size(2) > 0,
              "batch, seq_len and n_heads must be positive");
  TORCH_CHECK(TQ.size(0) <= INT32_MAX && TQ.size(1) <= INT32_MAX && TQ.size(2) <= INT32_MAX,
              "tensor dimension too large");

  at::Tensor TO;
  if (out_.has_value() && out_->defined()) {
    TO = out_.value();
    AFA_CHECK_CUDA(TO);
    AFA_CHECK_LAST_DIM(TO);
    TORCH_CHECK(TO.dtype() == TQ.dtype(), "Output tensor must have the same dtype as inputs");
    TORCH_CHECK(TQ.sizes() == TO.sizes(), "Query and output tensors have same shape");
    TORCH_CHECK(TO.device() == TQ.device(), "Output tensor must be on the same device");
  } else {
    TO = at::empty_like(TQ, at::MemoryFormat::Contiguous);
  }

  const float runtime = launch(TQ, TK, TV, TO, dt, 0.f /* 1/sqrt(d_head), as the reference */,
                               false, nullptr, benchmark);
  return std::make_tuple(TO, static_cast<double>(runtime));
}

// Fills AfaFwdArgs from the tensors and launches on the current stream; with
// `benchmark`, times the launch with CUDA events and checks the status word.
float launch(const at::Tensor& TQ, const at::Tensor& TK, const at::Tensor& TV, const at::Tensor& TO,
             int dt, float scale, bool causal, float* lse, bool benchmark) {
  AfaFwdArgs args{};
  args.q = TQ.data_ptr();
  args.k = TK.data_ptr();
  args.v = TV.data_ptr();
  args.o = TO.data_ptr();
  const at::Tensor* ts[4] = {&TQ, &TK, &TV, &TO};
  int64_t* ss[4] = {args.q_strides, args.k_strides, args.v_strides, args.o_strides};
  for (int t = 0; t < 4; ++t)
    for (int d = 0; d < 3; ++d) ss[t][d] = ts[t]->stride(d);
  args.batch = static_cast<int32_t>(TQ.size(0));
  args.seq_len = static_cast<int32_t>(TQ.size(1));
  args.n_heads = static_cast<int32_t>(TQ.size(2));
  args.head_dim = static_cast<int32_t>(TQ.size(3));
  args.dtype = dt;
  args.scale = scale;
  args.status = status_word(TQ.device().index()).device;
  {
    std::lock_guard<std::mutex> lock(g_test_mu);
    args.test_flags = g_test_flags;
    args.timeout_ns = g_test_timeout_ns;
    g_test_flags = 0;
    g_test_timeout_ns = 0;
  }
  args.seq_len_kv = static_cast<int32_t>(TK.size(1));
  args.n_kv_heads = static_cast<int32_t>(TK.size(2));
  args.causal = causal ? 1 : 0;
  args.lse = lse;

  cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  args.sched = causal ? sched_words(TQ.device(), stream) : nullptr;
  float runtime = 0.f;
  cudaEvent_t start = nullptr, stop = nullptr;
  if (benchmark) {
    TORCH_CHECK(cudaEventCreate(&start) == cudaSuccess && cudaEventCreate(&stop) == cudaSuccess,
                "cudaEventCreate failed");
    cudaEventRecord(start, stream);
  }
  const int rc = afa_fwd_sm100(&args, stream);
  if (benchmark) {
    cudaEventRecord(stop, stream);
    cudaEventSynchronize(stop);
    cudaEventElapsedTime(&runtime, start, stop);
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
  }
  TORCH_CHECK(rc == AFA_OK, "afa_fwd_sm100 failed: ", afa_strerror(rc));
  if (benchmark) {  // the launch has finished: its own status is in the word
    const int32_t st = take_status(TQ.device().index());
    TORCH_CHECK(st == 0, "attention kernel reported: ", afa_status_string(st));
  }
  return runtime;
}

// Beyond the reference: q [B, N, H, d]; k, v [B, N_kv, H_kv, d] with H_kv
// dividing H; optional causal mask (bottom-right aligned); optional fp32
// log-sum-exp [B, H, N].  Returns (O, lse or None).
std::tuple<at::Tensor, std::optional<at::Tensor>> forward_ext(
    const at::Tensor& TQ, const at::Tensor& TK, const at::Tensor& TV, std::optional<at::Tensor> out_,
    bool causal, std::optional<double> softmax_scale, bool return_lse) {
  AFA_CHECK_CUDA(TQ);
  AFA_CHECK_CUDA(TK);
  AFA_CHECK_CUDA(TV);
  AFA_CHECK_LAST_DIM(TQ);
  AFA_CHECK_LAST_DIM(TK);
  AFA_CHECK_LAST_DIM(TV);
  c10::cuda::CUDAGuard device_guard{TQ.device()};
  const int dev = TQ.device().index();
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  TORCH_CHECK(major == 10 && minor == 0,
              "Flash Attention (sm_100a build) requires SM_100 (current: SM_", major, ".", minor,
              ")");
  raise_earlier_abort(dev);
  const int dt = dtype_code(TQ);
  TORCH_CHECK(dt > 0, "Only fp16 and bf16 are supported");
  TORCH_CHECK(TK.dtype() == TQ.dtype() && TV.dtype() == TQ.dtype(),
              "Input tensors must have the same data type");
  TORCH_CHECK(TK.device() == TQ.device() && TV.device() == TQ.device(),
              "Input tensors must be on the same device");
  TORCH_CHECK(afa_fwd_sm100_supported(dt, static_cast<int32_t>(TQ.size(3))) == 1,
              "no sm_100a kernel for head_dim ", TQ.size(3), " (64 and 128 are compiled)");
  TORCH_CHECK(TK.sizes() == TV.sizes(), "key and value tensors must have the same shape");
  TORCH_CHECK(TK.size(0) == TQ.size(0), "query and key batch sizes differ");
  TORCH_CHECK(TK.size(3) == TQ.size(3), "query and key head_dim differ");
  TORCH_CHECK(TQ.size(0) > 0 && TQ.size(1) > 0 && TQ.size(2) > 0 && TK.size(1) > 0 && TK.size(2) > 0,
              "batch, seq_len and n_heads must be positive");
  TORCH_CHECK(TQ.size(2) % TK.size(2) == 0, "the number of query heads (", TQ.size(2),
              ") must be a multiple of the number of key/value heads (", TK.size(2), ")");
  TORCH_CHECK(TQ.size(0) <= INT32_MAX && TQ.size(1) <= INT32_MAX && TQ.size(2) <= INT32_MAX &&
                  TK.size(1) <= INT32_MAX,
              "tensor dimension too large");
  double scale = 0.0;
  if (softmax_scale.has_value()) {
    scale = softmax_scale.value();
    TORCH_CHECK(scale > 0.0, "softmax_scale must be positive");
  }
  at::Tensor TO;
  if (out_.has_value() && out_->defined()) {
    TO = out_.value();
    AFA_CHECK_CUDA(TO);
    AFA_CHECK_LAST_DIM(TO);
    TORCH_CHECK(TO.dtype() == TQ.dtype(), "Output tensor must have the same dtype as inputs");
    TORCH_CHECK(TQ.sizes() == TO.sizes(), "Query and output tensors have same shape");
    TORCH_CHECK(TO.device() == TQ.device(), "Output tensor must be on the same device");
  } else {
    TO = at::empty_like(TQ, at::MemoryFormat::Contiguous);
  }
  std::optional<at::Tensor> lse;
  if (return_lse)
    lse = at::empty({TQ.size(0), TQ.size(2), TQ.size(1)},
                    at::TensorOptions().dtype(at::kFloat).device(TQ.device()));
  launch(TQ, TK, TV, TO, dt, static_cast<float>(scale), causal,
         lse.has_value() ? lse->data_ptr<float>() : nullptr, false);
  return std::make_tuple(TO, lse);
}

// Host-resident inputs and output: q [B, N, H, d], k, v [B, N_kv, H_kv, d] and O
// in host memory (contiguous; page-locked for the copies to overlap).  The batch
// is split into `chunks` slices that flow through two sets of device buffers on
// three streams: while the kernel runs on slice c (the current stream), slice
// c+1 is copied in and slice c-1 copied out, so the transfers over the host link
// overlap each other and the compute.  Stream-ordered: returns after queuing;
// the current stream is ordered after the last copy out.  Returns O (host).
at::Tensor forward_host(const at::Tensor& HQ, const at::Tensor& HK, const at::Tensor& HV,
                        std::optional<at::Tensor> out_, bool causal, int64_t chunks) {
  for (const at::Tensor* t : {&HQ, &HK, &HV}) {
    TORCH_CHECK(t->device().is_cpu(), "forward_host takes host (CPU) tensors");
    TORCH_CHECK(t->dim() == 4 && t->is_contiguous(), "inputs must be contiguous [batch, seq, heads, head_dim]");
  }
  const int dt = dtype_code(HQ);
  TORCH_CHECK(dt > 0, "Only fp16 and bf16 are supported");
  TORCH_CHECK(HK.dtype() == HQ.dtype() && HV.dtype() == HQ.dtype(), "Input tensors must have the same data type");
  TORCH_CHECK(HK.sizes() == HV.sizes(), "key and value tensors must have the same shape");
  TORCH_CHECK(HK.size(0) == HQ.size(0) && HK.size(3) == HQ.size(3), "query and key batch / head_dim differ");
  TORCH_CHECK(HQ.size(0) > 0 && HQ.size(1) > 0 && HQ.size(2) > 0 && HK.size(1) > 0 && HK.size(2) > 0,
              "batch, seq_len and n_heads must be positive");
  TORCH_CHECK(HQ.size(2) % HK.size(2) == 0, "the number of query heads (", HQ.size(2),
              ") must be a multiple of the number of key/value heads (", HK.size(2), ")");
  TORCH_CHECK(afa_fwd_sm100_supported(dt, static_cast<int32_t>(HQ.size(3))) == 1,
              "no sm_100a kernel for head_dim ", HQ.size(3), " (64 and 128 are compiled)");
  at::Tensor HO;
  if (out_.has_value() && out_->defined()) {
    HO = out_.value();
    TORCH_CHECK(HO.device().is_cpu() && HO.is_contiguous() && HO.sizes() == HQ.sizes() && HO.dtype() == HQ.dtype(),
                "o must be a contiguous host tensor shaped and typed like q");
    // A copy into pageable memory returns only when it has finished, which
    // would hold each slice's copy in behind the previous slice's kernel.
    TORCH_CHECK(HO.is_pinned(), "o must be page-locked (pin_memory()) so its copies overlap the compute");
  } else {
    HO = at::empty(HQ.sizes(), HQ.options().pinned_memory(true));
  }
  const int dev = c10::cuda::current_device();
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  TORCH_CHECK(major == 10 && minor == 0,
              "Flash Attention (sm_100a build) requires SM_100 (current: SM_", major, ".", minor, ")");
  raise_earlier_abort(dev);

  const int64_t B = HQ.size(0);
  // Default 16 slices: at [16, 8192, 32, 128] only the first slice's copy in and
  // the last one's copy out stay exposed (63 ms per call against 58 ms for the
  // 3.2 GB of inputs alone at 55.6 GB/s host-to-device).
  const int64_t n_chunks = std::max<int64_t>(1, std::min<int64_t>(chunks > 0 ? chunks : 16, B));
  const int64_t per = (B + n_chunks - 1) / n_chunks;  // batches per slice
  const auto dopt = HQ.options().device(at::kCUDA, dev).pinned_memory(false);
  auto slice_shape = [&](const at::Tensor& t) {
    std::vector<int64_t> sz(t.sizes().begin(), t.sizes().end());
    sz[0] = per;
    return sz;
  };
  at::Tensor dq[2], dk[2], dv[2], dout[2];
  for (int i = 0; i < 2; ++i) {
    dq[i] = at::empty(slice_shape(HQ), dopt);
    dk[i] = at::empty(slice_shape(HK), dopt);
    dv[i] = at::empty(slice_shape(HV), dopt);
    dout[i] = at::empty(slice_shape(HQ), dopt);
  }
  c10::cuda::CUDAStream comp = at::cuda::getCurrentCUDAStream();
  c10::cuda::CUDAStream h2d = c10::cuda::getStreamFromPool(false, static_cast<c10::DeviceIndex>(dev));
  c10::cuda::CUDAStream d2h = c10::cuda::getStreamFromPool(false, static_cast<c10::DeviceIndex>(dev));
  // Events destroyed on every exit path, including an error thrown mid-loop.
  struct Event {
    cudaEvent_t e = nullptr;
    Event() {
      TORCH_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess, "cudaEventCreate failed");
    }
    ~Event() {
      if (e != nullptr) cudaEventDestroy(e);
    }
    Event(const Event&) = delete;
    Event& operator=(const Event&) = delete;
    operator cudaEvent_t() const { return e; }
  };
  Event start, h2d_done[2], comp_done[2], d2h_done[2];
  // The buffers were taken from the current stream's pool: earlier work on it
  // completes before the copy stream writes them.
  cudaEventRecord(start, comp.stream());
  cudaStreamWaitEvent(h2d.stream(), start, 0);
  const size_t esz = HQ.element_size();
  auto row_bytes = [&](const at::Tensor& t) { return static_cast<size_t>(t.numel() / t.size(0)) * esz; };
  for (int64_t c = 0; c < n_chunks; ++c) {
    const int64_t b0 = c * per;
    if (b0 >= B) break;
    const int64_t nb = std::min(per, B - b0);
    const int s = static_cast<int>(c & 1);
    // in: slice c -> buffer set s, after the kernel of slice c-2 has read it
    if (c >= 2) cudaStreamWaitEvent(h2d.stream(), comp_done[s], 0);
    const at::Tensor* hs[3] = {&HQ, &HK, &HV};
    at::Tensor* ds[3] = {&dq[s], &dk[s], &dv[s]};
    for (int t = 0; t < 3; ++t) {
      const size_t rb = row_bytes(*hs[t]);
      TORCH_CHECK(cudaMemcpyAsync(ds[t]->data_ptr(), static_cast<const char*>(hs[t]->data_ptr()) + b0 * rb, nb * rb,
                                  cudaMemcpyHostToDevice, h2d.stream()) == cudaSuccess,
                  "host-to-device copy failed");
    }
    cudaEventRecord(h2d_done[s], h2d.stream());
    // compute: after the slice is in and buffer set s's previous O has been copied out
    cudaStreamWaitEvent(comp.stream(), h2d_done[s], 0);
    if (c >= 2) cudaStreamWaitEvent(comp.stream(), d2h_done[s], 0);
    launch(dq[s].narrow(0, 0, nb), dk[s].narrow(0, 0, nb), dv[s].narrow(0, 0, nb), dout[s].narrow(0, 0, nb), dt, 0.f,
           causal, nullptr, false);
    cudaEventRecord(comp_done[s], comp.stream());
    // out: O of slice c
    cudaStreamWaitEvent(d2h.stream(), comp_done[s], 0);
    const size_t rb = row_bytes(HQ);
    TORCH_CHECK(cudaMemcpyAsync(static_cast<char*>(HO.data_ptr()) + b0 * rb, dout[s].data_ptr(), nb * rb,
                                cudaMemcpyDeviceToHost, d2h.stream()) == cudaSuccess,
                "device-to-host copy failed");
    cudaEventRecord(d2h_done[s], d2h.stream());
  }
  // The current stream (and with it the buffers' reuse) follows the last copies.
  for (int i = 0; i < 2; ++i) {
    cudaStreamWaitEvent(comp.stream(), d2h_done[i], 0);
    cudaStreamWaitEvent(comp.stream(), h2d_done[i], 0);
  }
  // The copies are still in flight when this returns.  Page-locked tensors from
  // torch's host allocator are told which stream uses them, so a caller that drops
  // them now (q.pin_memory() passed as a temporary) does not get their memory
  // handed to a new tensor before the copies have read or written it -- what
  // torch's own non-blocking copy_ does.  Pageable memory needs nothing: the
  // runtime stages it before cudaMemcpyAsync returns.
  auto keep_until_copied = [](const at::Tensor& t, const c10::cuda::CUDAStream& s) {
    if (t.is_pinned())
      at::getHostAllocator(at::kCUDA)->record_event(t.storage().mutable_data(),
                                                    t.storage().data_ptr().get_context(), s.unwrap());
  };
  keep_until_copied(HQ, h2d);
  keep_until_copied(HK, h2d);
  keep_until_copied(HV, h2d);
  keep_until_copied(HO, d2h);
  return HO;
}

// Waits for all work on `device`, then takes (and clears) its status word;
// raises RuntimeError if a kernel since the last check reported an error.
void check_status(int64_t device) {
  const at::Device dev(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  c10::cuda::CUDAGuard g{dev};
  TORCH_CHECK(cudaDeviceSynchronize() == cudaSuccess, "cudaDeviceSynchronize failed");
  const int32_t st = take_status(static_cast<int>(device));
  TORCH_CHECK(st == 0, "attention kernel reported: ", afa_status_string(st));
}

// Test hook: the next launch of this module runs with these AFA_TEST_* flags
// and wait bound (nanoseconds, 0 = default); later launches are normal again.
void set_test_flags(int64_t flags, int64_t timeout_ns) {
  TORCH_CHECK(flags >= 0 && timeout_ns >= 0, "flags and timeout_ns must be non-negative");
  std::lock_guard<std::mutex> lock(g_test_mu);
  g_test_flags = static_cast<uint32_t>(flags);
  g_test_timeout_ns = static_cast<uint64_t>(timeout_ns);
}

std::vector<std::tuple<int, int>> kernel_keys() {
  std::vector<std::tuple<int, int>> out;
  for (int dt : {AFA_DTYPE_FP16, AFA_DTYPE_BF16})
    for (int d : {64, 128})
      if (afa_fwd_sm100_supported(dt, d)) out.emplace_back(dt, d);
  return out;
}

// Raises a RuntimeError whose message is formatted from integers -- the same
// error path as the shape/config checks above; lets the CPU tests verify that
// C++ exceptions cross the binding intact.
void raise_formatted_error(int64_t a, int64_t b) {
  TORCH_CHECK(false, "formatted error ", a, " / ", b);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &flash_attention_forward, py::arg("kernel_cfg"), py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("o") = py::none(), py::arg("benchmark") = false,
        "Flash Attention forward (CUDA, sm_100a)");
  m.def("forward_ext", &forward_ext, py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("o") = py::none(), py::arg("causal") = false, py::arg("softmax_scale") = py::none(),
        py::arg("return_lse") = false,
        "Attention forward with K/V of their own length and head count (GQA), an optional causal "
        "mask (bottom-right aligned) and an optional fp32 log-sum-exp [batch, heads, seq]");
  m.def("forward_host", &forward_host, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o") = py::none(),
        py::arg("causal") = false, py::arg("chunks") = 0,
        "Attention forward on host tensors: batch slices copied in, computed and copied out on three "
        "streams so the transfers overlap each other and the compute (pinned host memory); returns O");
  m.def("check_status", &check_status, py::arg("device") = 0,
        "Wait for `device`, then raise RuntimeError if a kernel on it reported an error since the last check");
  m.def("_set_test_flags", &set_test_flags, py::arg("flags"), py::arg("timeout_ns") = 0,
        "Test hook: AFA_TEST_* flags and wait bound for the next launch only");
  m.def("_raise_formatted_error", &raise_formatted_error, py::arg("a"), py::arg("b"));
  m.def("kernel_keys", &kernel_keys, "(dtype code, d_head) pairs with a compiled sm_100a kernel");
}
