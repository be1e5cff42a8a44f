// dcn_abi.cu -- the extern "C" entry points declared in include/dcn_b200.h:
// argument checks, workspace carving and dispatch to the kernel families
// (tensor-core kernels where they apply, SIMT kernels otherwise).
//
// Error behaviour mirrors the reference host code
// (mps_deform_conv/csrc/deform_conv2d_mps.mm:597-657): the same checks, the same
// messages, reported through a status code and dcn_last_error() instead of a
// C++ exception.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "dcn_internal.h"
#include "dcn_tc.h"

namespace dcn {

static thread_local std::string g_last_error;
static std::atomic<unsigned long long> g_launches{0};

void note_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

// ---------------------------------------------------------------- profiling
struct ProfRecord {
  const char* name;
  cudaEvent_t start, stop;
};
static std::atomic<bool> g_prof_on{false};
static std::mutex g_prof_mu;
static std::vector<ProfRecord> g_prof;
static std::vector<cudaEvent_t> g_event_pool;

static cudaEvent_t prof_event() {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

KernelScope::KernelScope(const char* name, cudaStream_t st) : name_(name), st_(st) {
  note_launch();
  nvtxRangePushA(name);  // host-side range around the launch, named after the kernel
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return;
  start_ = prof_event();
  if (start_ && cudaEventRecord(start_, st) != cudaSuccess) start_ = nullptr;
}

KernelScope::~KernelScope() {
  nvtxRangePop();
  if (!start_) return;
  cudaEvent_t stop = prof_event();
  if (!stop || cudaEventRecord(stop, st_) != cudaSuccess) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof.push_back({name_, start_, stop});
}

static int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

static int cuda_fail(cudaError_t e, const char* where) {
  return fail(DCN_ERR_CUDA, "%s: CUDA error %d (%s)", where, (int)e, cudaGetErrorString(e));
}

static int ok() {
  g_last_error.clear();
  return DCN_OK;
}

// Output extent with floor division, as the reference's Python layer computes
// it (mps_deform_conv/__init__.py:208-209): a padded input smaller than the
// dilated kernel gives a non-positive extent and is rejected.
static long long out_extent(long long in, long long pad, long long dil, long long k, long long stride) {
  const long long num = in + 2 * pad - (dil * (k - 1) + 1);
  const long long q = num >= 0 ? num / stride : -((-num + stride - 1) / stride);
  return q + 1;
}

static size_t elem_size(int dtype) { return dtype == DCN_FLOAT32 ? 4 : 2; }

static int validate(const dcn_conv_desc* d) {
  if (!d) return fail(DCN_ERR_INVALID_ARGUMENT, "descriptor is NULL");
  if (d->dtype != DCN_FLOAT32 && d->dtype != DCN_FLOAT16 && d->dtype != DCN_BFLOAT16)
    return fail(DCN_ERR_UNSUPPORTED, "dtype %d is not one of float32, float16, bfloat16", d->dtype);
  if (d->stride_h <= 0 || d->stride_w <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "stride must be positive, got stride=(%lld, %lld)",
                (long long)d->stride_h, (long long)d->stride_w);
  if (d->dilation_h <= 0 || d->dilation_w <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "dilation must be positive, got dilation=(%lld, %lld)",
                (long long)d->dilation_h, (long long)d->dilation_w);
  if (d->pad_h < 0 || d->pad_w < 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "padding must be non-negative, got padding=(%lld, %lld)",
                (long long)d->pad_h, (long long)d->pad_w);
  if (d->kernel_h <= 0 || d->kernel_w <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "kernel_size must be positive, got kernel=(%lld, %lld)",
                (long long)d->kernel_h, (long long)d->kernel_w);
  if (d->n_weight_grps <= 0) return fail(DCN_ERR_INVALID_ARGUMENT, "n_weight_grps must be positive");
  if (d->n_offset_grps <= 0) return fail(DCN_ERR_INVALID_ARGUMENT, "n_offset_grps must be positive");
  if (d->batch < 0 || d->in_channels <= 0 || d->in_h <= 0 || d->in_w <= 0 || d->out_channels <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT,
                "tensor sizes must be positive (batch may be 0): batch=%lld in_channels=%lld "
                "in_h=%lld in_w=%lld out_channels=%lld",
                (long long)d->batch, (long long)d->in_channels, (long long)d->in_h,
                (long long)d->in_w, (long long)d->out_channels);
  if (d->in_channels % d->n_weight_grps != 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "in_channels (%lld) must be divisible by n_weight_grps (%lld)",
                (long long)d->in_channels, (long long)d->n_weight_grps);
  if (d->out_channels % d->n_weight_grps != 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "out_channels (%lld) must be divisible by n_weight_grps (%lld)",
                (long long)d->out_channels, (long long)d->n_weight_grps);
  if (d->in_channels % d->n_offset_grps != 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "in_channels (%lld) must be divisible by n_offset_grps (%lld)",
                (long long)d->in_channels, (long long)d->n_offset_grps);
  const long long out_h = out_extent(d->in_h, d->pad_h, d->dilation_h, d->kernel_h, d->stride_h);
  const long long out_w = out_extent(d->in_w, d->pad_w, d->dilation_w, d->kernel_w, d->stride_w);
  if (out_h <= 0 || out_w <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT,
                "Invalid output dimensions: out_h=%lld, out_w=%lld. Check stride/padding/dilation values.",
                out_h, out_w);
  const long long lim = 2147483647LL;
  const long long num_kernels = d->in_channels * out_h * out_w * d->batch;
  if (num_kernels > lim)
    return fail(DCN_ERR_UNSUPPORTED, "num_kernels (%lld) exceeds int32 limit. Reduce tensor dimensions.", num_kernels);
  if (d->in_channels * d->kernel_h * d->kernel_w > lim)
    return fail(DCN_ERR_UNSUPPORTED, "column_height (%lld) exceeds int32 limit. Reduce tensor dimensions.",
                (long long)(d->in_channels * d->kernel_h * d->kernel_w));
  if (d->batch * out_h * out_w > lim)
    return fail(DCN_ERR_UNSUPPORTED, "column_width (%lld) exceeds int32 limit. Reduce tensor dimensions.",
                (long long)(d->batch * out_h * out_w));
  if (d->in_h * d->in_w > lim)
    return fail(DCN_ERR_UNSUPPORTED, "in_h*in_w (%lld) exceeds int32 limit. Reduce tensor dimensions.",
                (long long)(d->in_h * d->in_w));
  if (d->out_channels * (d->in_channels / d->n_weight_grps) * d->kernel_h * d->kernel_w > lim)
    return fail(DCN_ERR_UNSUPPORTED, "weight numel exceeds int32 limit");
  return DCN_OK;
}

// Workspace layout of the fused backward on the SIMT kernels.
struct SimtBwdLayout {
  size_t gcol, gin32, gw32, goff, total;
};
static SimtBwdLayout simt_bwd_layout(const dcn_conv_desc* d, const Geom& g) {
  SimtBwdLayout L;
  const bool f32 = d->dtype == DCN_FLOAT32;
  size_t off = 0;
  L.gcol = off;  off += ws_align(sizeof(float) * (size_t)g.C * g.T * (size_t)g.P);
  // fp32 grad_input accumulator: NCHW for fp16/bf16 on the scalar scatter,
  // channels-last for the four-channel scatter (every dtype)
  L.gin32 = off; off += ws_align(sizeof(float) * (size_t)g.B * g.C * g.H * g.W);
  L.gw32 = off;  off += f32 ? 0 : ws_align(sizeof(float) * (size_t)g.Co * g.Cig * g.T);
  L.goff = off;  off += ws_align(elem_size(d->dtype) * (size_t)g.B * g.OG * 2 * g.T * g.HWo);
  L.total = off;
  return L;
}

template <typename F>
static int dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case DCN_FLOAT32: return f((float*)nullptr);
    case DCN_FLOAT16: return f((__half*)nullptr);
    default: return f((__nv_bfloat16*)nullptr);
  }
}

}  // namespace dcn

using namespace dcn;

extern "C" {

int dcn_abi_version(void) { return 100; }

uint64_t dcn_launch_count(void) { return (uint64_t)g_launches.load(std::memory_order_relaxed); }

void dcn_profile_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (enable) {  // a new recording starts: recycle the previous one's events
    for (auto& r : g_prof) {
      g_event_pool.push_back(r.start);
      g_event_pool.push_back(r.stop);
    }
    g_prof.clear();
  }
  g_prof_on.store(enable != 0, std::memory_order_relaxed);
}

int dcn_profile_summary(int max_entries, char* names, size_t name_stride, uint64_t* launches,
                        double* total_ms) {
  std::vector<ProfRecord> recs;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    recs = g_prof;
  }
  std::vector<std::string> keys;
  std::vector<uint64_t> cnt;
  std::vector<double> ms;
  for (auto& r : recs) {
    if (cudaEventSynchronize(r.stop) != cudaSuccess) return -1;
    float t = 0.f;
    if (cudaEventElapsedTime(&t, r.start, r.stop) != cudaSuccess) return -1;
    size_t i = 0;
    while (i < keys.size() && keys[i] != r.name) ++i;
    if (i == keys.size()) {
      keys.push_back(r.name);
      cnt.push_back(0);
      ms.push_back(0.0);
    }
    cnt[i] += 1;
    ms[i] += t;
  }
  const int n = (int)keys.size() < max_entries ? (int)keys.size() : max_entries;
  for (int i = 0; i < n; ++i) {
    if (names && name_stride) {
      strncpy(names + (size_t)i * name_stride, keys[i].c_str(), name_stride - 1);
      names[(size_t)i * name_stride + name_stride - 1] = 0;
    }
    if (launches) launches[i] = cnt[i];
    if (total_ms) total_ms[i] = ms[i];
  }
  return (int)keys.size();
}

const char* dcn_last_error(void) { return g_last_error.c_str(); }

int dcn_validate(const dcn_conv_desc* desc) {
  int r = validate(desc);
  return r == DCN_OK ? ok() : r;
}

int dcn_output_size(const dcn_conv_desc* d, int64_t* out_h, int64_t* out_w) {
  if (!d || !out_h || !out_w) return fail(DCN_ERR_INVALID_ARGUMENT, "NULL argument");
  if (d->stride_h <= 0 || d->stride_w <= 0) return fail(DCN_ERR_INVALID_ARGUMENT, "stride must be positive");
  *out_h = out_extent(d->in_h, d->pad_h, d->dilation_h, d->kernel_h, d->stride_h);
  *out_w = out_extent(d->in_w, d->pad_w, d->dilation_w, d->kernel_w, d->stride_w);
  if (*out_h <= 0 || *out_w <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT,
                "Invalid output dimensions: out_h=%lld, out_w=%lld. Check stride/padding/dilation values.",
                (long long)*out_h, (long long)*out_w);
  return ok();
}

int dcn_uses_tensor_cores(const dcn_conv_desc* d) {
  if (validate(d) != DCN_OK) return 0;
  return tc_forward_supported(*d, make_geom(*d)) ? 1 : 0;
}

size_t dcn_forward_workspace_size(const dcn_conv_desc* d) {
  if (validate(d) != DCN_OK) return 0;
  const Geom g = make_geom(*d);
  return tc_forward_supported(*d, g) ? tc_forward_workspace(*d, g) : simt_forward_workspace(g);
}

static int forward_impl(const dcn_conv_desc* d, const void* input, const void* weight,
                        const void* offset, const void* mask, const void* bias, void* output,
                        void* saved, size_t saved_bytes, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int r = validate(d);
  if (r != DCN_OK) return r;
  const Geom g = make_geom(*d);
  if (g.P == 0) return ok();
  if (!input || !weight || !offset || !output || (d->use_mask && !mask))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer (input, weight, offset, output%s)",
                d->use_mask ? ", mask" : "");
  cudaStream_t st = (cudaStream_t)stream;
  if (tc_forward_supported(*d, g)) {
    const size_t need = tc_forward_workspace(*d, g);
    if (workspace_bytes < need || (need && !workspace))
      return fail(DCN_ERR_WORKSPACE, "forward workspace too small: need %zu bytes, got %zu", need,
                  workspace_bytes);
    const size_t need_saved = saved ? saved_layout(g).total : 0;
    if (saved && saved_bytes < need_saved)
      return fail(DCN_ERR_WORKSPACE, "saved state too small: need %zu bytes, got %zu", need_saved, saved_bytes);
    cudaError_t e = tc_forward(*d, g, input, weight, false, offset, mask, bias, output, workspace, saved, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_forward (tensor core)");
  }
  const size_t need = simt_forward_workspace(g);
  if (workspace_bytes < need || (need && !workspace))
    return fail(DCN_ERR_WORKSPACE, "forward workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
  // training: the columns go to the saved state (the backward's weight
  // gradient reads them there) instead of the workspace
  const size_t need_saved = saved ? simt_saved_columns_bytes(g) : 0;
  if (saved && saved_bytes < need_saved)
    return fail(DCN_ERR_WORKSPACE, "saved state too small: need %zu bytes, got %zu", need_saved, saved_bytes);
  void* cols = saved && need_saved ? saved : (need ? workspace : nullptr);
  cudaError_t e = cudaSuccess;
  dispatch_dtype(d->dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    e = simt_forward<T>(g, (const T*)input, (const T*)weight, (const T*)offset,
                        (const T*)(d->use_mask ? mask : nullptr), (const T*)bias, (T*)output, cols, st);
    return 0;
  });
  return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_forward");
}

int dcn_deform_conv2d_forward(const dcn_conv_desc* d, const void* input, const void* weight,
                              const void* offset, const void* mask, const void* bias, void* output,
                              void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(d, input, weight, offset, mask, bias, output, nullptr, 0, workspace,
                      workspace_bytes, stream);
}

size_t dcn_saved_state_bytes(const dcn_conv_desc* d) {
  if (validate(d) != DCN_OK) return 0;
  const Geom g = make_geom(*d);
  if (tc_backward_supported(*d, g)) return saved_layout(g).total;
  // both passes on the SIMT kernels: the forward's fp32 columns
  return tc_forward_supported(*d, g) ? 0 : simt_saved_columns_bytes(g);
}

int dcn_deform_conv2d_forward_train(const dcn_conv_desc* d, const void* input, const void* weight,
                                    const void* offset, const void* mask, const void* bias,
                                    void* output, void* saved, size_t saved_bytes, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (validate(d) != DCN_OK) return validate(d);
  if (dcn_saved_state_bytes(d) == 0) saved = nullptr;
  return forward_impl(d, input, weight, offset, mask, bias, output, saved, saved_bytes, workspace,
                      workspace_bytes, stream);
}

int dcn_deformable_im2col(const dcn_conv_desc* d0, const void* input, const void* offset,
                          const void* mask, void* columns, void* stream) {
  dcn_conv_desc dd = *d0;
  dd.out_channels = dd.n_weight_grps;  // unused by this call
  int r = validate(&dd);
  if (r != DCN_OK) return r;
  const Geom g = make_geom(dd);
  if (g.P == 0) return ok();
  if (!input || !offset || !columns || (dd.use_mask && !mask))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  cudaError_t e = cudaSuccess;
  dispatch_dtype(dd.dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    e = simt_im2col<T>(g, (const T*)input, (const T*)offset, (const T*)(dd.use_mask ? mask : nullptr),
                       (T*)columns, (cudaStream_t)stream);
    return 0;
  });
  return e == cudaSuccess ? ok() : cuda_fail(e, "deformable_im2col");
}

size_t dcn_backward_input_workspace_size(const dcn_conv_desc* d) {
  if (validate(d) != DCN_OK) return 0;
  const Geom g = make_geom(*d);
  return d->dtype == DCN_FLOAT32 ? 0 : ws_align(sizeof(float) * (size_t)g.B * g.C * g.H * g.W);
}

int dcn_deform_conv2d_backward_input(const dcn_conv_desc* d0, const void* grad_col,
                                     const void* offset, const void* mask, void* grad_input,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  dcn_conv_desc dd = *d0;
  dd.out_channels = dd.n_weight_grps;
  int r = validate(&dd);
  if (r != DCN_OK) return r;
  const Geom g = make_geom(dd);
  cudaStream_t st = (cudaStream_t)stream;
  const long long n = (long long)g.B * g.C * g.H * g.W;
  if (n == 0) return ok();
  if (!grad_col || !offset || !grad_input || (dd.use_mask && !mask))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  const size_t need = dcn_backward_input_workspace_size(&dd);
  if (workspace_bytes < need || (need && !workspace))
    return fail(DCN_ERR_WORKSPACE, "backward_input workspace too small: need %zu bytes, got %zu", need,
                workspace_bytes);
  cudaError_t e = cudaSuccess;
  dispatch_dtype(dd.dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    float* acc = need ? (float*)workspace : (float*)grad_input;
    if ((e = cudaMemsetAsync(acc, 0, sizeof(float) * (size_t)n, st)) != cudaSuccess) return 0;
    if ((e = simt_col2im<T, T>(g, (const T*)grad_col, (const T*)offset,
                               (const T*)(dd.use_mask ? mask : nullptr), acc, st)) != cudaSuccess)
      return 0;
    if (need) e = convert_f32<T>(acc, (T*)grad_input, n, st);
    return 0;
  });
  return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward_input");
}

int dcn_deform_conv2d_backward_offset_mask(const dcn_conv_desc* d0, const void* grad_col,
                                           const void* input, const void* offset, const void* mask,
                                           void* grad_offset, void* grad_mask, void* stream) {
  dcn_conv_desc dd = *d0;
  dd.out_channels = dd.n_weight_grps;
  int r = validate(&dd);
  if (r != DCN_OK) return r;
  const Geom g = make_geom(dd);
  if (g.P == 0) return ok();
  if (!grad_col || !input || !offset || !grad_offset || (dd.use_mask && (!mask || !grad_mask)))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  cudaError_t e = cudaSuccess;
  dispatch_dtype(dd.dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    e = simt_col2im_coord<T, T>(g, (const T*)grad_col, (const T*)input, (const T*)offset,
                                (const T*)(dd.use_mask ? mask : nullptr), (T*)grad_offset,
                                (T*)(dd.use_mask ? grad_mask : nullptr), (cudaStream_t)stream);
    return 0;
  });
  return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward_offset_mask");
}

size_t dcn_backward_workspace_size(const dcn_conv_desc* d) {
  if (validate(d) != DCN_OK) return 0;
  const Geom g = make_geom(*d);
  if (tc_backward_supported(*d, g)) return tc_backward_workspace(*d, g);
  return simt_bwd_layout(d, g).total;
}

// `ready(user)`, when given, is called once the grad_weight / grad_bias
// kernels are enqueued (dcn_deform_conv2d_backward_overlap).
static int backward_impl(const dcn_conv_desc* d, const void* grad_output, const void* input,
                         const void* weight, const void* offset, const void* mask,
                         const void* saved, size_t saved_bytes, void* grad_input,
                         void* grad_weight, void* grad_offset, void* grad_mask, void* grad_bias,
                         void* workspace, size_t workspace_bytes, void* stream,
                         dcn_params_ready_fn ready = nullptr, void* user = nullptr) {
  int r = validate(d);
  if (r != DCN_OK) return r;
  const Geom g = make_geom(*d);
  cudaStream_t st = (cudaStream_t)stream;
  if (!d->use_mask) grad_mask = nullptr;
  if (g.P == 0) {  // empty batch: parameter gradients are zero sums
    cudaError_t e = cudaSuccess;
    const size_t es = elem_size(d->dtype);
    if (grad_weight) e = cudaMemsetAsync(grad_weight, 0, es * (size_t)g.Co * g.Cig * g.T, st);
    if (e == cudaSuccess && grad_bias) e = cudaMemsetAsync(grad_bias, 0, es * (size_t)g.Co, st);
    if (e == cudaSuccess && ready) ready(user);
    return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward");
  }
  if (!grad_output || !input || !weight || !offset || (d->use_mask && !mask))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer (grad_output, input, weight, offset%s)",
                d->use_mask ? ", mask" : "");
  if (tc_backward_supported(*d, g)) {
    const size_t need = tc_backward_workspace(*d, g);
    if (workspace_bytes < need || (need && !workspace))
      return fail(DCN_ERR_WORKSPACE, "backward workspace too small: need %zu bytes, got %zu", need,
                  workspace_bytes);
    if (saved && saved_bytes < saved_layout(g).total)
      return fail(DCN_ERR_WORKSPACE, "saved state too small: need %zu bytes, got %zu", saved_layout(g).total,
                  saved_bytes);
    cudaError_t e = tc_backward(*d, g, grad_output, input, weight, offset, mask, saved, grad_input,
                                grad_weight, grad_offset, grad_mask, grad_bias, workspace, st, ready, user);
    return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward (tensor core)");
  }
  const SimtBwdLayout L = simt_bwd_layout(d, g);
  if (workspace_bytes < L.total || !workspace)
    return fail(DCN_ERR_WORKSPACE, "backward workspace too small: need %zu bytes, got %zu", L.total,
                workspace_bytes);
  char* base = (char*)workspace;
  const bool f32 = d->dtype == DCN_FLOAT32;
  SimtBackwardWs ws;
  ws.gcol = (float*)(base + L.gcol);
  ws.gin32 = f32 ? nullptr : (float*)(base + L.gin32);
  ws.gacc = (float*)(base + L.gin32);
  ws.gw32 = f32 ? nullptr : (float*)(base + L.gw32);
  ws.goff_scratch = base + L.goff;
  if (saved) {
    const size_t need_saved = simt_saved_columns_bytes(g);
    if (saved_bytes < need_saved)
      return fail(DCN_ERR_WORKSPACE, "saved state too small: need %zu bytes, got %zu", need_saved, saved_bytes);
    if (need_saved) ws.cols = static_cast<const float*>(saved);
  }
  cudaError_t e = cudaSuccess;
  dispatch_dtype(d->dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    e = simt_backward<T>(g, (const T*)grad_output, (const T*)input, (const T*)weight,
                         (const T*)offset, (const T*)(d->use_mask ? mask : nullptr), (T*)grad_input,
                         (T*)grad_weight, (T*)grad_offset, (T*)grad_mask, (T*)grad_bias, ws, st);
    return 0;
  });
  if (e == cudaSuccess && ready) ready(user);
  return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward");
}

int dcn_deform_conv2d_backward(const dcn_conv_desc* d, const void* grad_output, const void* input,
                               const void* weight, const void* offset, const void* mask,
                               void* grad_input, void* grad_weight, void* grad_offset,
                               void* grad_mask, void* grad_bias, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return backward_impl(d, grad_output, input, weight, offset, mask, nullptr, 0, grad_input, grad_weight,
                       grad_offset, grad_mask, grad_bias, workspace, workspace_bytes, stream);
}

int dcn_deform_conv2d_backward_train(const dcn_conv_desc* d, const void* grad_output,
                                     const void* input, const void* weight, const void* offset,
                                     const void* mask, const void* saved, size_t saved_bytes,
                                     void* grad_input, void* grad_weight, void* grad_offset,
                                     void* grad_mask, void* grad_bias, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (validate(d) != DCN_OK) return validate(d);
  if (dcn_saved_state_bytes(d) == 0) saved = nullptr;
  return backward_impl(d, grad_output, input, weight, offset, mask, saved, saved_bytes, grad_input,
                       grad_weight, grad_offset, grad_mask, grad_bias, workspace, workspace_bytes,
                       stream);
}

int dcn_deform_conv2d_backward_overlap(const dcn_conv_desc* d, const void* grad_output,
                                       const void* input, const void* weight, const void* offset,
                                       const void* mask, const void* saved, size_t saved_bytes,
                                       void* grad_input, void* grad_weight, void* grad_offset,
                                       void* grad_mask, void* grad_bias, void* workspace,
                                       size_t workspace_bytes, void* stream, dcn_params_ready_fn params_ready,
                                       void* user_data) {
  if (validate(d) != DCN_OK) return validate(d);
  if (dcn_saved_state_bytes(d) == 0) saved = nullptr;
  return backward_impl(d, grad_output, input, weight, offset, mask, saved, saved_bytes, grad_input,
                       grad_weight, grad_offset, grad_mask, grad_bias, workspace, workspace_bytes,
                       stream, params_ready, user_data);
}

// ---------------------------------------------------------------- layouts and the DCNv2 head
// dcn_ex_options: channels-last input / output and the DCNv2 head layout
// (offset_mask [B][OG*T*3][Ho][Wo]: offsets in channels [0, 2*OG*T), mask
// logits in [2*OG*T, 3*OG*T); the kernels read both in place and apply the
// sigmoid).  Anything but NCHW without the head needs the tensor-core path;
// the head also needs 32-channel dgrad slabs.
static bool plain_options(const dcn_ex_options* o) {
  return !o || (o->input_layout == DCN_LAYOUT_NCHW && o->output_layout == DCN_LAYOUT_NCHW && !o->head && !o->flags);
}

static Geom ex_geom(const dcn_conv_desc& d, const dcn_ex_options* o) {
  Geom g = make_geom(d);
  if (o && o->head) {
    g.off_bs = 3LL * g.OG * g.T * g.HWo;
    g.msk_bs = g.off_bs;
    g.msk_logit = 1;
  }
  g.in_nhwc = o && o->input_layout == DCN_LAYOUT_NHWC;
  g.out_nhwc = o && o->output_layout == DCN_LAYOUT_NHWC;
  return g;
}

int dcn_ex_supported(const dcn_conv_desc* d, const dcn_ex_options* o, int backward) {
  if (validate(d) != DCN_OK) return 0;
  if (plain_options(o)) return 1;
  if ((o->input_layout != DCN_LAYOUT_NCHW && o->input_layout != DCN_LAYOUT_NHWC) ||
      (o->output_layout != DCN_LAYOUT_NCHW && o->output_layout != DCN_LAYOUT_NHWC) || (o->head != 0 && o->head != 1) ||
      (o->flags & ~DCN_EX_WEIGHT_IMAGE) || ((o->flags & DCN_EX_WEIGHT_IMAGE) && backward))
    return 0;
  const Geom g = ex_geom(*d, o);
  if (o->head && (!d->use_mask || g.cpo % 32 != 0 || (long long)g.B * g.H * g.W * g.C >= (1LL << 31) ||
                  !tc_backward_supported(*d, g)))
    return 0;
  return (backward ? tc_backward_supported(*d, g) : tc_forward_supported(*d, g)) ? 1 : 0;
}

size_t dcn_weight_image_bytes(const dcn_conv_desc* d) {
  const dcn_ex_options o = {DCN_LAYOUT_NCHW, DCN_LAYOUT_NCHW, 0, DCN_EX_WEIGHT_IMAGE};
  if (!dcn_ex_supported(d, &o, 0)) return 0;
  return elem_size(d->dtype) * (size_t)d->out_channels * (size_t)(d->in_channels / d->n_weight_grps) *
         (size_t)(d->kernel_h * d->kernel_w);
}

int dcn_weight_image(const dcn_conv_desc* d, const void* weight, void* image, size_t image_bytes, void* stream) {
  const size_t need = dcn_weight_image_bytes(d);
  if (!need)
    return fail(DCN_ERR_UNSUPPORTED, "weight_image: the problem does not run on the tensor-core forward");
  if (!weight || !image) return fail(DCN_ERR_INVALID_ARGUMENT, "weight_image: NULL weight or image");
  if (image_bytes < need)
    return fail(DCN_ERR_WORKSPACE, "weight image too small: need %zu bytes, got %zu", need, image_bytes);
  if ((reinterpret_cast<uintptr_t>(image) & 15) != 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "the weight image must be 16-byte aligned");
  const Geom g = make_geom(*d);
  cudaError_t e = tc_weight_image(*d, g, weight, image, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "weight_image");
}

int dcn_head_supported(const dcn_conv_desc* d) {
  const dcn_ex_options o = {DCN_LAYOUT_NCHW, DCN_LAYOUT_NCHW, 1, 0};
  return dcn_ex_supported(d, &o, 1);
}

static int ex_check(const dcn_conv_desc* d, const dcn_ex_options* o, int backward, const char* fn) {
  const int r = validate(d);
  if (r != DCN_OK) return r;
  if (!dcn_ex_supported(d, o, backward))
    return fail(DCN_ERR_UNSUPPORTED,
                "%s: channels-last layouts, the DCNv2 head layout and weight images need fp16/bf16 with "
                "per-group channels that the tensor-core kernels take (the head layout also needs use_mask and "
                "offset groups of a multiple of 32 channels; a weight image serves forward calls only)",
                fn);
  return DCN_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int dcn_deform_conv2d_forward_ex(const dcn_conv_desc* d, const dcn_ex_options* o, const void* input,
                                 const void* weight, const void* offset, const void* mask, const void* bias,
                                 void* output, void* saved, size_t saved_bytes, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (plain_options(o))
    return forward_impl(d, input, weight, offset, mask, bias, output,
                        dcn_saved_state_bytes(d) ? saved : nullptr, saved_bytes, workspace, workspace_bytes, stream);
  int r = ex_check(d, o, 0, "deform_conv2d_forward_ex");
  if (r != DCN_OK) return r;
  const Geom g = ex_geom(*d, o);
  if (g.P == 0) return ok();
  if (!input || !weight || !offset || !output || (d->use_mask && !o->head && !mask))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer (input, weight, offset, output%s)",
                d->use_mask && !o->head ? ", mask" : "");
  if ((g.in_nhwc && !aligned16(input)) || (g.out_nhwc && !aligned16(output)))
    return fail(DCN_ERR_INVALID_ARGUMENT, "channels-last input and output must be 16-byte aligned");
  const size_t need = tc_forward_workspace(*d, g);
  if (workspace_bytes < need || (need && !workspace))
    return fail(DCN_ERR_WORKSPACE, "forward workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
  if (saved && saved_bytes < saved_layout(g).total)
    return fail(DCN_ERR_WORKSPACE, "saved state too small: need %zu bytes, got %zu", saved_layout(g).total,
                saved_bytes);
  const bool image = (o->flags & DCN_EX_WEIGHT_IMAGE) != 0;
  if (image && saved)
    return fail(DCN_ERR_INVALID_ARGUMENT, "a weight image serves forward-only calls: saved must be NULL");
  if (image && !aligned16(weight))
    return fail(DCN_ERR_INVALID_ARGUMENT, "the weight image must be 16-byte aligned");
  if (o->head)
    mask = static_cast<const char*>(offset) + elem_size(d->dtype) * (size_t)2 * g.OG * g.T * g.HWo;
  cudaError_t e = tc_forward(*d, g, input, weight, image, offset, mask, bias, output, workspace, saved,
                             (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_forward_ex");
}

int dcn_deform_conv2d_backward_ex(const dcn_conv_desc* d, const dcn_ex_options* o, const void* grad_output,
                                  const void* input, const void* weight, const void* offset, const void* mask,
                                  const void* saved, size_t saved_bytes, void* grad_input, void* grad_weight,
                                  void* grad_offset, void* grad_mask, void* grad_bias, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (plain_options(o))
    return dcn_deform_conv2d_backward_train(d, grad_output, input, weight, offset, mask, saved, saved_bytes,
                                            grad_input, grad_weight, grad_offset, grad_mask, grad_bias, workspace,
                                            workspace_bytes, stream);
  int r = ex_check(d, o, 1, "deform_conv2d_backward_ex");
  if (r != DCN_OK) return r;
  const Geom g = ex_geom(*d, o);
  cudaStream_t st = (cudaStream_t)stream;
  if (g.P == 0) {  // empty batch: parameter gradients are zero sums
    cudaError_t e = cudaSuccess;
    const size_t es = elem_size(d->dtype);
    if (grad_weight) e = cudaMemsetAsync(grad_weight, 0, es * (size_t)g.Co * g.Cig * g.T, st);
    if (e == cudaSuccess && grad_bias) e = cudaMemsetAsync(grad_bias, 0, es * (size_t)g.Co, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward_ex");
  }
  if (!grad_output || !input || !weight || !offset || (d->use_mask && !o->head && !mask))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer (grad_output, input, weight, offset%s)",
                d->use_mask && !o->head ? ", mask" : "");
  if (g.in_nhwc && !aligned16(input))
    return fail(DCN_ERR_INVALID_ARGUMENT, "channels-last input must be 16-byte aligned");
  const size_t need = tc_backward_workspace(*d, g);
  if (workspace_bytes < need || (need && !workspace))
    return fail(DCN_ERR_WORKSPACE, "backward workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
  if (saved && saved_bytes < saved_layout(g).total)
    return fail(DCN_ERR_WORKSPACE, "saved state too small: need %zu bytes, got %zu", saved_layout(g).total,
                saved_bytes);
  if (o->head) {
    mask = static_cast<const char*>(offset) + elem_size(d->dtype) * (size_t)2 * g.OG * g.T * g.HWo;
    grad_mask = nullptr;  // grad_offset holds the whole head gradient
  }
  if (!d->use_mask) grad_mask = nullptr;
  cudaError_t e = tc_backward(*d, g, grad_output, input, weight, offset, mask, saved, grad_input, grad_weight,
                              grad_offset, grad_mask, grad_bias, workspace, st, nullptr, nullptr);
  return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward_ex");
}

int dcn_deform_conv2d_forward_head(const dcn_conv_desc* d, const void* input, const void* weight,
                                   const void* offset_mask, const void* bias, void* output, void* saved,
                                   size_t saved_bytes, void* workspace, size_t workspace_bytes, void* stream) {
  if (validate(d) != DCN_OK) return validate(d);
  if (!dcn_head_supported(d))
    return fail(DCN_ERR_UNSUPPORTED, "deform_conv2d_forward_head: the DCNv2 head layout needs use_mask, fp16/bf16, "
                                     "per-group channels that the tensor-core kernels take and offset groups of a "
                                     "multiple of 32 channels");
  const dcn_ex_options o = {DCN_LAYOUT_NCHW, DCN_LAYOUT_NCHW, 1, 0};
  return dcn_deform_conv2d_forward_ex(d, &o, input, weight, offset_mask, nullptr, bias, output, saved, saved_bytes,
                                      workspace, workspace_bytes, stream);
}

int dcn_deform_conv2d_backward_head(const dcn_conv_desc* d, const void* grad_output, const void* input,
                                    const void* weight, const void* offset_mask, const void* saved,
                                    size_t saved_bytes, void* grad_input, void* grad_weight,
                                    void* grad_offset_mask, void* grad_bias, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (validate(d) != DCN_OK) return validate(d);
  if (!dcn_head_supported(d))
    return fail(DCN_ERR_UNSUPPORTED, "deform_conv2d_backward_head: the DCNv2 head layout needs use_mask, fp16/bf16, "
                                     "per-group channels that the tensor-core kernels take and offset groups of a "
                                     "multiple of 32 channels");
  const dcn_ex_options o = {DCN_LAYOUT_NCHW, DCN_LAYOUT_NCHW, 1, 0};
  return dcn_deform_conv2d_backward_ex(d, &o, grad_output, input, weight, offset_mask, nullptr, saved, saved_bytes,
                                       grad_input, grad_weight, grad_offset_mask, nullptr, grad_bias, workspace,
                                       workspace_bytes, stream);
}

int dcn_deform_conv2d_backward_input_noalloc(const dcn_conv_desc* d0, const void* grad_col,
                                             const void* offset, const void* mask,
                                             void* grad_input, void* stream) {
  dcn_conv_desc dd = *d0;
  dd.out_channels = dd.n_weight_grps;
  int r = validate(&dd);
  if (r != DCN_OK) return r;
  const Geom g = make_geom(dd);
  const long long n = (long long)g.B * g.C * g.H * g.W;
  // fp32 accumulates in grad_input itself; only fp16/bf16 use the fixed array
  if (dd.dtype != DCN_FLOAT32 && n > noalloc_max_elems())
    return fail(DCN_ERR_UNSUPPORTED,
                "backward_input_noalloc: grad_input has %lld elements, more than the %lld this "
                "allocation-free entry point supports for fp16/bf16; use "
                "dcn_deform_conv2d_backward_input with a workspace",
                n, noalloc_max_elems());
  if (n == 0) return ok();
  if (!grad_col || !offset || !grad_input || (dd.use_mask && !mask))
    return fail(DCN_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  cudaError_t e = noalloc_backward_input_dispatch(dd.dtype, g, grad_col, offset,
                                                  dd.use_mask ? mask : nullptr, grad_input,
                                                  (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "deform_conv2d_backward_input_noalloc");
}

int dcn_debug_bounds_enabled(void) {
#ifdef DCN_DEBUG_BOUNDS
  return 1;
#else
  return 0;
#endif
}

int dcn_debug_bounds_read(dcn_bounds_record* out, int reset) {
  if (!out) return fail(DCN_ERR_INVALID_ARGUMENT, "dcn_debug_bounds_read: out is NULL");
  dcn::DebugBounds acc = {};
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = dcn::debug_bounds_collect_tc(&acc, reset != 0);
  if (e == cudaSuccess) e = dcn::debug_bounds_collect_tc_bwd(&acc, reset != 0);
  if (e == cudaSuccess) e = dcn::debug_bounds_collect_simt(&acc, reset != 0);
  if (e != cudaSuccess) return cuda_fail(e, "dcn_debug_bounds_read");
  out->count = acc.count;
  out->index = acc.index;
  out->extent = acc.extent;
  out->site = acc.site;
  out->width = acc.width;
  return ok();
}

int dcn_device_status(void* stream) {
  int v = 0;
  cudaError_t e = tc_read_and_clear_status(&v, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "dcn_device_status");
  if (v != 0) return fail(DCN_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait expired (code %d)", v);
  return ok();
}

}  // extern "C"
