// dcn_capi.cu -- extern "C" entry points of libdcn_b200 (declared in
// include/dcn_b200.h): argument validation with the reference's messages,
// workspace carving and kernel dispatch.  No entry point allocates device
// memory or synchronises the host.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "dcn_launch.h"
#include "dcn_b200.h"
#include "dcn_kernels.h"
#include "dcn_tc.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(DCN_ERR_CUDA, "%s: CUDA error %d (%s)", where, (int)e, cudaGetErrorString(e));
}

#define DCN_CHECK(cond, ...)                                  \
  do {                                                        \
    if (!(cond)) return fail(DCN_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

// ---- kernel profiler: a CUDA event pair around every launch when enabled --
// (tracing for the bench and for users; off by default, one branch per
// launch when off).
struct ProfRecord {
  const char* name;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof_recs;
std::vector<cudaEvent_t> g_prof_pool;

cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

struct ProfScope {
  const char* name;
  cudaStream_t stream;
  cudaEvent_t start = nullptr;
  ProfScope(const char* n, cudaStream_t s) : name(n), stream(s) {
    if (!g_prof_on) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    start = prof_event();
    if (start) cudaEventRecord(start, stream);
  }
  void done() {
    if (!start) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    cudaEvent_t stop = prof_event();
    if (stop) {
      cudaEventRecord(stop, stream);
      g_prof_recs.push_back({name, start, stop});
    } else {
      g_prof_pool.push_back(start);
    }
  }
};

#define DCN_CUDA(expr, where)                             \
  do {                                                    \
    ProfScope ps_(where, stream);                         \
    cudaError_t e_ = (expr);                              \
    ps_.done();                                           \
    if (e_ != cudaSuccess) return cuda_fail(e_, where);   \
  } while (0)

#define DCN_CUDA_ON(strm, expr, where)                    \
  do {                                                    \
    ProfScope ps_(where, strm);                           \
    cudaError_t e_ = (expr);                              \
    ps_.done();                                           \
    if (e_ != cudaSuccess) return cuda_fail(e_, where);   \
  } while (0)

// Stream-ordering calls (no kernel, not profiled).
#define DCN_ORDER(expr, where)                            \
  do {                                                    \
    cudaError_t e_ = (expr);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, where);   \
  } while (0)

// ---- side streams for independent helper kernels ----
// Per device, two non-blocking streams and their events, created on first
// use.  A call forks them from the caller's stream with an event and joins
// them back before the work that needs their results, so the ordering holds
// under CUDA graph capture too (make the first call before capturing: it
// creates the streams).  The mutex keeps one call's fork/join sequence from
// interleaving with another host thread's on the shared events.
struct SideStreams {
  cudaStream_t s[2] = {nullptr, nullptr};
  cudaEvent_t fork = nullptr, join[2] = {nullptr, nullptr};
};
std::mutex g_side_mu;
std::map<int, SideStreams> g_side;

SideStreams* side_streams_locked() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  auto it = g_side.find(dev);
  if (it != g_side.end()) return &it->second;
  SideStreams ss;
  bool ok = cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) == cudaSuccess;
  for (int i = 0; i < 2 && ok; ++i)
    ok = cudaStreamCreateWithFlags(&ss.s[i], cudaStreamNonBlocking) == cudaSuccess &&
         cudaEventCreateWithFlags(&ss.join[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    return nullptr;  // everything stays on the caller's stream
  }
  return &(g_side[dev] = ss);
}

class Fork {
 public:
  // `use` false: everything stays on the caller's stream
  Fork(cudaStream_t main, bool use)
      : lk_(g_side_mu), ss_(use ? side_streams_locked() : nullptr), main_(main) {}
  cudaStream_t side(int i) const { return ss_ ? ss_->s[i] : main_; }
  // side streams start after everything enqueued on the caller's stream so far
  cudaError_t fork() {
    if (!ss_) return cudaSuccess;
    cudaError_t e = cudaEventRecord(ss_->fork, main_);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(ss_->s[i], ss_->fork, 0);
    return e;
  }
  // the caller's stream continues after side stream i's work so far
  cudaError_t join(int i) {
    if (!ss_) return cudaSuccess;
    cudaError_t e = cudaEventRecord(ss_->join[i], ss_->s[i]);
    return e == cudaSuccess ? cudaStreamWaitEvent(main_, ss_->join[i], 0) : e;
  }

 private:
  std::unique_lock<std::mutex> lk_;
  SideStreams* ss_;
  cudaStream_t main_;
};

// The side streams pay when the helpers beside the input staging are large
// enough to hide the cross-stream event waits: inputs of 16 MB and more (the
// detection neck's 31 MB); below that the waits cost more than the overlap.
bool side_streams_pay(const dcn::Geom& g) {
  return (long long)g.N * g.C * g.HW * (long long)sizeof(float) >= (16LL << 20);
}

bool is_device_ptr(const void* p) {
  if (p == nullptr) return false;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

int num_sms_current() { return dcn::device_sm_count(); }

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Carves aligned sub-buffers out of the caller's workspace.
struct Carver {
  char* base;
  size_t used = 0;
  explicit Carver(void* p) : base(static_cast<char*>(p)) {}
  float* take(size_t nfloats) {
    float* p = reinterpret_cast<float*>(base + used);
    used += align_up(nfloats * sizeof(float));
    return p;
  }
};

// DCN_TEST_WAIT_TIMEOUT: the tensor-core kernels' TMA producers issue
// nothing and every wait gives up after a short budget.
void apply_test_flags(dcn::Geom& g, uint32_t flags) {
  if (flags & DCN_TEST_WAIT_TIMEOUT) {
    g.no_async = 1;
    g.wait_limit = dcn::kTestWaitLimit;
  }
}

// Validation shared by forward and backward (.mm:202-267, :693-760).
int make_geom(const dcn_shape* s, bool use_mask, bool use_bias, dcn::Geom& g,
              const char* op) {
  DCN_CHECK(s != nullptr, "%s: shape must not be NULL", op);
  DCN_CHECK(s->batch >= 0 && s->in_channels >= 0 && s->height >= 0 && s->width >= 0 &&
                s->out_channels >= 0,
            "%s: tensor dimensions must be non-negative", op);
  DCN_CHECK(s->kernel_h > 0 && s->kernel_w > 0, "kernel dims must be positive");
  DCN_CHECK(s->groups > 0, "groups must be positive, got %lld", (long long)s->groups);
  DCN_CHECK(s->stride_h > 0 && s->stride_w > 0, "stride must be positive");
  DCN_CHECK(s->dilation_h > 0 && s->dilation_w > 0, "dilation must be positive");
  DCN_CHECK(s->pad_h >= 0 && s->pad_w >= 0, "padding must be non-negative");
  DCN_CHECK(s->in_channels % s->groups == 0, "channels (%lld) not divisible by groups (%lld)",
            (long long)s->in_channels, (long long)s->groups);
  DCN_CHECK(s->out_channels % s->groups == 0,
            "out_channels (%lld) not divisible by groups (%lld)", (long long)s->out_channels,
            (long long)s->groups);
  const int64_t Ho = (s->height + 2 * s->pad_h - s->dilation_h * (s->kernel_h - 1) - 1) / s->stride_h + 1;
  const int64_t Wo = (s->width + 2 * s->pad_w - s->dilation_w * (s->kernel_w - 1) - 1) / s->stride_w + 1;
  DCN_CHECK(Ho > 0 && Wo > 0, "calculated output size (%lldx%lld) is non-positive",
            (long long)Ho, (long long)Wo);
  DCN_CHECK(s->deformable_groups > 0, "deformable_groups must be positive, got %lld",
            (long long)s->deformable_groups);
  DCN_CHECK(s->in_channels % s->deformable_groups == 0,
            "channels (%lld) not divisible by deformable_groups (%lld)",
            (long long)s->in_channels, (long long)s->deformable_groups);
  const int64_t kk = s->kernel_h * s->kernel_w;
  const int64_t lim = (int64_t)1 << 31;
  // per-image element counts are indexed in int32 inside the kernels
  if (s->in_channels * s->height * s->width >= lim || s->out_channels * Ho * Wo >= lim ||
      2 * s->deformable_groups * kk * Ho * Wo >= lim || s->batch * Ho * Wo >= lim ||
      s->out_channels * (s->in_channels / s->groups) * kk >= lim || s->height * s->width > 65535LL * 32)
    return fail(DCN_ERR_UNSUPPORTED, "%s: per-image tensor sizes beyond 2^31 elements are not supported", op);
  g.N = (int)s->batch; g.C = (int)s->in_channels; g.H = (int)s->height; g.W = (int)s->width;
  g.outC = (int)s->out_channels; g.kh = (int)s->kernel_h; g.kw = (int)s->kernel_w;
  g.sh = (int)s->stride_h; g.sw = (int)s->stride_w; g.ph = (int)s->pad_h; g.pw = (int)s->pad_w;
  g.dh = (int)s->dilation_h; g.dw = (int)s->dilation_w;
  g.G = (int)s->groups; g.dg = (int)s->deformable_groups;
  g.Ho = (int)Ho; g.Wo = (int)Wo;
  g.use_mask = use_mask ? 1 : 0; g.use_bias = use_bias ? 1 : 0;
  g.mask_logits = 0;
  g.oy0 = 0;
  g.wait_limit = dcn::kWaitLimit;
  g.no_async = 0;
  g.Cg = g.C / g.G; g.Og = g.outC / g.G; g.cpg = g.dg ? g.C / g.dg : 0;
  g.kk = g.kh * g.kw; g.P = g.Ho * g.Wo; g.HW = g.H * g.W;
  g.NP = (long long)g.N * g.P;
  return DCN_OK;
}

int fwd_cpad(const dcn::Geom& g) { return dcn::ceil_div(g.Cg, 8) * 8; }

enum class FwdAlgo { kDirect, kGemm, kTc, kDgroup };

// TF32 and 3xTF32 run the tensor-core kernels; 3xTF32 splits every operand.
bool tc_math(uint32_t flags) {
  const uint32_t m = flags & 0xff;
  return m == DCN_MATH_TF32 || m == DCN_MATH_3XTF32;
}
bool split_math(uint32_t flags) { return (flags & 0xff) == DCN_MATH_3XTF32; }

FwdAlgo pick_fwd(const dcn::Geom& g, uint32_t flags) {
  if (flags & DCN_ALGO_SIMT_GEMM) return FwdAlgo::kGemm;
  if (flags & DCN_ALGO_SIMT_DIRECT) return dcn::fwd_direct_supported(g) ? FwdAlgo::kDirect : FwdAlgo::kGemm;
  if (tc_math(flags) && dcn::tc_fwd_supported(g)) return FwdAlgo::kTc;
  if (dcn::dgroup_supported(g)) return FwdAlgo::kDgroup;
  if (dcn::fwd_direct_supported(g)) return FwdAlgo::kDirect;
  return FwdAlgo::kGemm;
}

// NHWC copy of the input plus one zero pixel row (C floats) at its end, the
// target of the tensor-core gathers' dropped corners.
size_t xt_floats(const dcn::Geom& g) { return (size_t)g.N * g.HW * g.C + g.C; }

// The least workspace the forward accepts (no staging copy of the input when
// the caller passes one, DCN_INPUT_STAGED).
size_t fwd_ws_min(const dcn::Geom& g, uint32_t flags) {
  size_t b = (flags & DCN_INPUT_STAGED) ? 0 : align_up(xt_floats(g) * sizeof(float));  // xt + zero row
  switch (pick_fwd(g, flags)) {
    case FwdAlgo::kGemm:
      b += align_up((size_t)g.G * g.kk * fwd_cpad(g) * g.Og * sizeof(float));
      break;
    case FwdAlgo::kTc:
      b += align_up(dcn::tc_fwd_weight_bytes(g, split_math(flags)));
      break;
    case FwdAlgo::kDirect:
    case FwdAlgo::kDgroup:
      break;
  }
  return b + kAlign;  // slack for aligning the caller's base pointer
}

// Scratch with which the tensor-core forward splits a short last round of
// tiles over all SMs.  The size query includes it; a workspace of only the
// minimum runs whole tiles (same results up to the order of fp32 sums).
size_t fwd_tail_ws(const dcn::Geom& g, uint32_t flags) {
  if (pick_fwd(g, flags) != FwdAlgo::kTc) return 0;
  return align_up(dcn::tc_fwd_tail_bytes(g, split_math(flags), false, num_sms_current()));
}

size_t fwd_ws(const dcn::Geom& g, uint32_t flags) { return fwd_ws_min(g, flags) + fwd_tail_ws(g, flags); }

// The fused tensor-core backward (grad columns, col2im, col2im_coord and the
// weight gradient in one kernel, no column buffer): TF32 with out channels
// per group <= 256, unless a weight-gradient route is pinned.
bool use_fused_bwd(const dcn::Geom& g, uint32_t flags) {
  return (flags & 0xff) == DCN_MATH_TF32 &&
         !(flags & (DCN_ALGO_SIMT_GEMM | DCN_ALGO_SIMT_DIRECT | DCN_ALGO_TC_GATHER_WEIGHT |
                    DCN_ALGO_TC_COLUMN_BUFFER)) &&
         dcn::tc_fused_supported(g);
}

// Tensor-core backward with the column buffer (weight gradient as a dense
// GEMM over the columns the grad-column kernel writes); DCN_ALGO_TC_GATHER_WEIGHT
// asks for the gather-based weight gradient where that kernel covers the shape.
bool use_col_path(const dcn::Geom& g, uint32_t flags) {
  return !use_fused_bwd(g, flags) && dcn::tc_wcol_supported(g, split_math(flags)) &&
         (!(flags & DCN_ALGO_TC_GATHER_WEIGHT) || !dcn::tc_wgather_supported(g));
}

bool use_tc_bwd(const dcn::Geom& g, uint32_t flags) {
  return tc_math(flags) && !(flags & (DCN_ALGO_SIMT_GEMM | DCN_ALGO_SIMT_DIRECT)) &&
         dcn::tc_bwd_supported(g) &&
         (use_fused_bwd(g, flags) || use_col_path(g, flags) || dcn::tc_wgather_supported(g));
}

size_t bwd_ws(const dcn::Geom& g, uint32_t flags) {
  size_t b = (flags & DCN_INPUT_STAGED) ? 0 : align_up(xt_floats(g) * sizeof(float));  // xt + zero row
  if (!(flags & DCN_INPUT_NHWC))
    b += align_up((size_t)g.N * g.HW * g.C * sizeof(float));           // grad x (NHWC)
  if (use_tc_bwd(g, flags)) {
    const size_t parts = split_math(flags) ? 2 : 1;                   // high (+ low) TF32 parts
    b += align_up(parts * g.N * g.outC * ((g.P + 3) & ~3) * sizeof(float));   // go_r
    b += align_up(parts * g.outC * g.Cg * g.kk * sizeof(float));               // packed weight
    b += align_up((size_t)g.outC * g.Cg * g.kk * sizeof(float));               // tap-major grad_weight
    if (use_col_path(g, flags))
      b += align_up(dcn::tc_col_bytes(g, split_math(flags)));                  // column buffer
    else if (!use_fused_bwd(g, flags))
      b += align_up(dcn::tc_plan_bytes(g));                                    // sampling plans
    else
      b += align_up(dcn::tc_bias_part_floats(g) * sizeof(float));              // bias partial sums
  } else {
    b += align_up((size_t)g.G * g.kk * g.Og * g.Cg * sizeof(float));   // packed weight
  }
  return b + kAlign;
}

void* align_ptr(void* p) {
  uintptr_t v = reinterpret_cast<uintptr_t>(p);
  return reinterpret_cast<void*>((v + kAlign - 1) / kAlign * kAlign);
}

}  // namespace

namespace dcn {
// Lets other translation units of the library report through dcn_last_error.
void set_last_error(int code, const char* msg) { fail(code, "%s", msg); }
// The least workspace dcn_forward accepts for this shape (0: invalid shape);
// dcn_forward_workspace_size adds the optional tail scratch.
size_t forward_min_workspace(const dcn_shape* s, uint32_t flags) {
  Geom g;
  if (make_geom(s, true, true, g, "dcn_forward_workspace_size") != DCN_OK) return 0;
  return fwd_ws_min(g, flags);
}
}  // namespace dcn

extern "C" {

DCN_API int dcn_abi_version(void) { return DCN_ABI_VERSION; }

DCN_API const char* dcn_last_error(void) { return g_last_error.c_str(); }

DCN_API int dcn_output_size(const dcn_shape* s, int64_t* out_h, int64_t* out_w) {
  dcn::Geom g;
  const int rc = make_geom(s, false, false, g, "dcn_output_size");
  if (rc != DCN_OK) return rc;
  if (out_h) *out_h = g.Ho;
  if (out_w) *out_w = g.Wo;
  return DCN_OK;
}

// Restricts a geometry to output rows [row0, row0 + rows) of every image:
// offset / mask / output / grad_output then hold those rows only; the input
// and grad_input stay whole.  rows < 0: the full output.
static int apply_rows(dcn::Geom& g, int64_t row0, int64_t rows, const char* op) {
  if (rows < 0) return DCN_OK;
  if (row0 < 0 || rows == 0 || row0 + rows > g.Ho)
    return fail(DCN_ERR_INVALID_ARGUMENT,
                "%s: output rows [%lld, %lld) outside the %d output rows", op, (long long)row0,
                (long long)(row0 + rows), g.Ho);
  g.oy0 = (int)row0;
  g.Ho = (int)rows;
  g.P = g.Ho * g.Wo;
  g.NP = (long long)g.N * g.P;
  return DCN_OK;
}

static size_t fwd_ws_rows(const dcn_shape* s, int64_t rows, uint32_t flags) {
  dcn::Geom g;
  if (make_geom(s, true, true, g, "dcn_forward_workspace_size") != DCN_OK) return 0;
  if (apply_rows(g, 0, rows, "dcn_forward_workspace_size") != DCN_OK) return 0;
  return fwd_ws(g, flags);
}

static size_t bwd_ws_rows(const dcn_shape* s, int64_t rows, uint32_t flags) {
  dcn::Geom g;
  if (make_geom(s, true, true, g, "dcn_backward_workspace_size") != DCN_OK) return 0;
  if (apply_rows(g, 0, rows, "dcn_backward_workspace_size") != DCN_OK) return 0;
  return bwd_ws(g, flags);
}

DCN_API size_t dcn_forward_workspace_size(const dcn_shape* s, uint32_t flags) {
  return fwd_ws_rows(s, -1, flags);
}

DCN_API size_t dcn_backward_workspace_size(const dcn_shape* s, uint32_t flags) {
  return bwd_ws_rows(s, -1, flags);
}

DCN_API size_t dcn_forward_rows_workspace_size(const dcn_shape* s, int64_t rows, uint32_t flags) {
  return rows > 0 ? fwd_ws_rows(s, rows, flags) : 0;
}

DCN_API size_t dcn_backward_rows_workspace_size(const dcn_shape* s, int64_t rows,
                                                uint32_t flags) {
  return rows > 0 ? bwd_ws_rows(s, rows, flags) : 0;
}

static int forward_core(const dcn_shape* s, int64_t row0, int64_t rows, const float* input,
                        const float* weight, const float* offset, const float* mask,
                        const float* bias, float* output, uint32_t flags, void* workspace,
                        size_t workspace_bytes, void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = make_geom(s, mask != nullptr, bias != nullptr, g, "deform_conv2d_forward");
  if (rc != DCN_OK) return rc;
  rc = apply_rows(g, row0, rows, "deform_conv2d_forward");
  if (rc != DCN_OK) return rc;
  g.mask_logits = (flags & DCN_MASK_LOGITS) && mask != nullptr ? 1 : 0;
  apply_test_flags(g, flags);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const long long out_numel = (long long)g.N * g.outC * g.P;
  if (out_numel == 0) return DCN_OK;  // .mm:273: nothing to dispatch
  auto dev_or_empty = [](const void* p, long long n) { return n == 0 || is_device_ptr(p); };
  DCN_CHECK(is_device_ptr(output), "deform_conv2d_forward: output must be a CUDA device buffer");
  DCN_CHECK(dev_or_empty(input, (long long)g.N * g.C * g.HW) &&
                dev_or_empty(offset, (long long)g.N * 2 * g.dg * g.kk * g.P) &&
                dev_or_empty(weight, (long long)g.outC * g.Cg * g.kk),
            "deform_conv2d_forward: input, weight and offset must be CUDA tensors");
  DCN_CHECK(mask == nullptr || is_device_ptr(mask), "mask must be a float32 CUDA tensor");
  DCN_CHECK(bias == nullptr || is_device_ptr(bias), "bias must be a float32 CUDA tensor");
  if (g.C == 0) {  // .mm:303-308: output is zeros (+ bias)
    DCN_CUDA(dcn::launch_fill_bias(output, g.use_bias ? bias : nullptr, g, stream), "fill");
    return DCN_OK;
  }
  const size_t need = fwd_ws_min(g, flags);
  if (workspace_bytes < need || workspace == nullptr)
    return fail(DCN_ERR_WORKSPACE, "deform_conv2d_forward: workspace of %zu bytes needed, %zu given",
                need, workspace_bytes);
  Carver ws(align_ptr(workspace));
  const size_t usable = workspace_bytes - (size_t)(ws.base - static_cast<char*>(workspace));
  // xt (+ its zero row): a transpose of NCHW input, a copy of NHWC input, or
  // the caller's staging copy (DCN_INPUT_STAGED: nothing to do).  It is the
  // workspace's first carve, where DCN_KEEP_STAGED leaves it for the caller.
  const bool staged = flags & DCN_INPUT_STAGED;
  DCN_CHECK(!(staged && (flags & DCN_KEEP_STAGED)),
            "deform_conv2d_forward: DCN_KEEP_STAGED needs an input to stage, not a staging copy");
  float* xt = staged ? const_cast<float*>(input) : ws.take(xt_floats(g));
  const FwdAlgo algo = pick_fwd(g, flags);
  const bool nhwc = flags & DCN_INPUT_NHWC;
  auto stage_input = [&]() {
    if (staged) return cudaSuccess;
    return nhwc ? dcn::launch_copy_nhwc(input, xt, g.N, g.C, g.HW, true, nullptr, stream)
                : dcn::launch_nchw_to_nhwc(input, xt, g.N, g.C, g.HW, true, nullptr, stream);
  };
  if (algo == FwdAlgo::kTc) {
    // the weight pack (side stream) runs beside the input transpose
    const bool split = split_math(flags);
    float* wt = ws.take(dcn::tc_fwd_weight_bytes(g, split) / sizeof(float));
    const int sms = num_sms_current();
    const size_t tail_bytes = dcn::tc_fwd_tail_bytes(g, split, false, sms);
    void* tail = tail_bytes > 0 && usable >= ws.used + tail_bytes ? ws.base + ws.used : nullptr;
    if (!staged && !nhwc && dcn::fwd_prologue_fits(input, xt, g)) {
      // the staging transpose and the weight pack in one launch
      DCN_CUDA(dcn::launch_fwd_prologue(input, xt, weight, wt, g, split, stream), "fwd_prologue");
    } else {
      Fork fk(stream, side_streams_pay(g) && !staged);
      DCN_ORDER(fk.fork(), "fork");
      DCN_CUDA_ON(fk.side(0), dcn::launch_tc_pack_weight(weight, wt, g, split, fk.side(0)),
                  "tc_pack_weight");
      if (!staged) DCN_CUDA(stage_input(), nhwc ? "copy_nhwc" : "nchw_to_nhwc");
      DCN_ORDER(fk.join(0), "join");
    }
    DCN_CUDA(dcn::launch_fwd_tc(g, xt, wt, offset, mask, bias, output, split, tail,
                                tail ? tail_bytes : 0, sms, stream),
             "fwd_tc");
    return DCN_OK;
  }
  if (!staged) DCN_CUDA(stage_input(), nhwc ? "copy_nhwc" : "nchw_to_nhwc");
  switch (algo) {
    case FwdAlgo::kDirect:
      DCN_CUDA(dcn::launch_fwd_simt_direct(g, xt, weight, offset, mask, bias, output, stream),
               "fwd_simt_direct");
      break;
    case FwdAlgo::kDgroup:
      DCN_CUDA(dcn::launch_fwd_dgroup(g, xt, weight, offset, mask, bias, output, stream),
               "fwd_dgroup");
      break;
    case FwdAlgo::kGemm: {
      const int cpad = fwd_cpad(g);
      float* wf = ws.take((size_t)g.G * g.kk * cpad * g.Og);
      DCN_CUDA(dcn::launch_pack_weight_fwd(weight, wf, g, cpad, stream), "pack_weight_fwd");
      DCN_CUDA(dcn::launch_fwd_simt_gemm(g, xt, wf, cpad, offset, mask, bias, output, stream),
               "fwd_simt_gemm");
      break;
    }
    case FwdAlgo::kTc:
      break;  // handled above
  }
  return DCN_OK;
}

}  // extern "C"

namespace {
bool use_bf16_tc(const dcn::Geom& g, uint32_t flags) {
  return g.C > 0 && !(flags & (DCN_ALGO_SIMT_GEMM | DCN_ALGO_SIMT_DIRECT)) &&
         dcn::tc_fwd_bf16_supported(g);
}
// fp32 copies of the operands for the upcast route: x, weight, offset, mask,
// bias, output (mask and bias counted whether present or not: an upper bound).
size_t bf16_upcast_bytes(const dcn::Geom& g) {
  return align_up((size_t)g.N * g.C * g.HW * 4) + align_up((size_t)g.outC * g.Cg * g.kk * 4) +
         align_up((size_t)g.N * 2 * g.dg * g.kk * g.P * 4) +
         align_up((size_t)g.N * g.dg * g.kk * g.P * 4) + align_up((size_t)g.outC * 4) +
         align_up((size_t)g.N * g.outC * g.P * 4);
}
// The least workspace of the 16-bit forward, and with the tail scratch of the
// tensor-core forward (the size query).
size_t fwd_bf16_ws_min(const dcn::Geom& g, uint32_t flags) {
  if (use_bf16_tc(g, flags))
    return align_up(((size_t)g.N * g.HW * g.C + g.C) * 2) +
           align_up(dcn::tc_fwd_weight_bf16_bytes(g)) + kAlign;
  return bf16_upcast_bytes(g) + kAlign + fwd_ws_min(g, flags);
}
size_t fwd_bf16_ws(const dcn::Geom& g, uint32_t flags) {
  if (use_bf16_tc(g, flags))
    return fwd_bf16_ws_min(g, flags) +
           align_up(dcn::tc_fwd_tail_bytes(g, false, true, num_sms_current()));
  return bf16_upcast_bytes(g) + kAlign + fwd_ws(g, flags);
}
}  // namespace

// The 16-bit forward, bf16 or fp16 (`f16`): the tensor-core kernel with
// 16-bit operands where it covers the shape, else the fp32 path on upcast
// copies with the output rounded back.
static int forward_h16(bool f16, const dcn_shape* s, const void* input, const void* weight,
                       const void* offset, const void* mask, const void* bias, void* output,
                       uint32_t flags, void* workspace, size_t workspace_bytes, void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = make_geom(s, mask != nullptr, bias != nullptr, g, "deform_conv2d_forward");
  if (rc != DCN_OK) return rc;
  g.mask_logits = (flags & DCN_MASK_LOGITS) && mask != nullptr ? 1 : 0;
  apply_test_flags(g, flags);
  const bool staged = flags & DCN_INPUT_STAGED, keep = flags & DCN_KEEP_STAGED;
  DCN_CHECK(!(staged && keep),
            "deform_conv2d_forward: DCN_KEEP_STAGED needs an input to stage, not a staging copy");
  DCN_CHECK(!(staged || keep) || use_bf16_tc(g, flags),
            "deform_conv2d_forward: a 16-bit staging copy needs the tensor-core forward, which "
            "does not cover this shape");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const long long out_numel = (long long)g.N * g.outC * g.P;
  if (out_numel == 0) return DCN_OK;
  const char* tname = f16 ? "float16" : "bfloat16";
  auto dev_or_empty = [](const void* p, long long n) { return n == 0 || is_device_ptr(p); };
  DCN_CHECK(is_device_ptr(output), "deform_conv2d_forward: output must be a CUDA device buffer");
  DCN_CHECK(dev_or_empty(input, (long long)g.N * g.C * g.HW) &&
                dev_or_empty(offset, (long long)g.N * 2 * g.dg * g.kk * g.P) &&
                dev_or_empty(weight, (long long)g.outC * g.Cg * g.kk),
            "deform_conv2d_forward: input, weight and offset must be CUDA tensors");
  DCN_CHECK(mask == nullptr || is_device_ptr(mask), "mask must be a %s CUDA tensor", tname);
  DCN_CHECK(bias == nullptr || is_device_ptr(bias), "bias must be a %s CUDA tensor", tname);
  const size_t need = fwd_bf16_ws_min(g, flags);
  if (workspace_bytes < need || workspace == nullptr)
    return fail(DCN_ERR_WORKSPACE, "deform_conv2d_forward: workspace of %zu bytes needed, %zu given",
                need, workspace_bytes);
  char* base = static_cast<char*>(align_ptr(workspace));
  if (use_bf16_tc(g, flags)) {
    // the 16-bit staging copy: the caller's (DCN_INPUT_STAGED) or the
    // workspace's first carve, where DCN_KEEP_STAGED leaves it
    void* xt = staged ? const_cast<void*>(input) : base;
    void* wt = base + (staged ? 0 : align_up(((size_t)g.N * g.HW * g.C + g.C) * 2));
    char* tail = static_cast<char*>(wt) + align_up(dcn::tc_fwd_weight_bf16_bytes(g));
    const int sms = num_sms_current();
    const size_t tail_bytes = dcn::tc_fwd_tail_bytes(g, false, true, sms);
    const size_t usable = workspace_bytes - (size_t)(tail - static_cast<char*>(workspace));
    if (tail_bytes == 0 || usable < tail_bytes) tail = nullptr;
    // the weight pack (side stream) runs beside the input staging
    Fork fk(stream, side_streams_pay(g) && !staged);
    DCN_ORDER(fk.fork(), "fork");
    DCN_CUDA_ON(fk.side(0), dcn::launch_tc_pack_weight_bf16(weight, wt, g, fk.side(0)),
                "tc_pack_weight");
    if (staged) {
      // nothing to stage
    } else if (flags & DCN_INPUT_NHWC) {  // channels-last: a copy plus the zero row
      const size_t xb = (size_t)g.N * g.HW * g.C * 2;
      if (xb) DCN_CUDA(cudaMemcpyAsync(xt, input, xb, cudaMemcpyDeviceToDevice, stream), "copy");
      DCN_CUDA(cudaMemsetAsync(static_cast<char*>(xt) + xb, 0, (size_t)g.C * 2, stream),
               "memset");
    } else {
      DCN_CUDA(dcn::launch_nchw_to_nhwc_bf16(input, xt, g.N, g.C, g.HW, /*zero_row=*/true,
                                             stream),
               "nchw_to_nhwc");
    }
    DCN_ORDER(fk.join(0), "join");
    DCN_CUDA(dcn::launch_fwd_tc_bf16(g, xt, wt, offset, mask, bias, output, f16, tail,
                                     tail ? tail_bytes : 0, sms, stream),
             f16 ? "fwd_tc_f16" : "fwd_tc_bf16");
    return DCN_OK;
  }
  // upcast route: fp32 copies, the fp32 forward, the result rounded back
  Carver ws(base);
  const long long nx = (long long)g.N * g.C * g.HW, nw = (long long)g.outC * g.Cg * g.kk;
  const long long noff = (long long)g.N * 2 * g.dg * g.kk * g.P;
  const long long nm = (long long)g.N * g.dg * g.kk * g.P;
  float* x32 = ws.take(nx);
  float* w32 = ws.take(nw);
  float* off32 = ws.take(noff);
  float* m32 = ws.take(nm);
  float* b32 = ws.take(g.outC);
  float* out32 = ws.take(out_numel);
  const char* up = f16 ? "f16_to_f32" : "bf16_to_f32";
  DCN_CUDA(dcn::launch_h16_to_f32(input, x32, nx, f16, stream), up);
  DCN_CUDA(dcn::launch_h16_to_f32(weight, w32, nw, f16, stream), up);
  DCN_CUDA(dcn::launch_h16_to_f32(offset, off32, noff, f16, stream), up);
  if (mask) DCN_CUDA(dcn::launch_h16_to_f32(mask, m32, nm, f16, stream), up);
  if (bias) DCN_CUDA(dcn::launch_h16_to_f32(bias, b32, g.outC, f16, stream), up);
  const size_t used = bf16_upcast_bytes(g);
  rc = dcn_forward(s, x32, w32, off32, mask ? m32 : nullptr, bias ? b32 : nullptr, out32, flags,
                   base + used, workspace_bytes - (size_t)(base - static_cast<char*>(workspace)) - used,
                   stream_);
  if (rc != DCN_OK) return rc;
  DCN_CUDA(dcn::launch_f32_to_h16(out32, output, out_numel, f16, stream),
           f16 ? "f32_to_f16" : "f32_to_bf16");
  return DCN_OK;
}

extern "C" {

DCN_API size_t dcn_forward_bf16_workspace_size(const dcn_shape* s, uint32_t flags) {
  dcn::Geom g;
  if (make_geom(s, true, true, g, "dcn_forward_bf16_workspace_size") != DCN_OK) return 0;
  return fwd_bf16_ws(g, flags);
}

DCN_API int dcn_forward_bf16(const dcn_shape* s, const void* input, const void* weight,
                             const void* offset, const void* mask, const void* bias,
                             void* output, uint32_t flags, void* workspace,
                             size_t workspace_bytes, void* stream) {
  return forward_h16(false, s, input, weight, offset, mask, bias, output, flags, workspace,
                     workspace_bytes, stream);
}

DCN_API size_t dcn_forward_f16_workspace_size(const dcn_shape* s, uint32_t flags) {
  dcn::Geom g;
  if (make_geom(s, true, true, g, "dcn_forward_f16_workspace_size") != DCN_OK) return 0;
  return fwd_bf16_ws(g, flags);
}

DCN_API int dcn_forward_f16(const dcn_shape* s, const void* input, const void* weight,
                            const void* offset, const void* mask, const void* bias, void* output,
                            uint32_t flags, void* workspace, size_t workspace_bytes,
                            void* stream) {
  return forward_h16(true, s, input, weight, offset, mask, bias, output, flags, workspace,
                     workspace_bytes, stream);
}

static int backward_core(const dcn_shape* s, int64_t row0, int64_t rows,
                         const float* grad_output, const float* input, const float* weight,
                         const float* offset, const float* mask, float* grad_input,
                         float* grad_offset, float* grad_mask, float* grad_weight,
                         float* grad_bias, uint32_t flags, void* workspace,
                         size_t workspace_bytes, void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = make_geom(s, mask != nullptr, grad_bias != nullptr, g, "deform_conv2d_backward");
  if (rc != DCN_OK) return rc;
  rc = apply_rows(g, row0, rows, "deform_conv2d_backward");
  if (rc != DCN_OK) return rc;
  g.mask_logits = (flags & DCN_MASK_LOGITS) && mask != nullptr ? 1 : 0;
  apply_test_flags(g, flags);
  DCN_CHECK(mask != nullptr || grad_mask == nullptr,
            "deform_conv2d_backward: grad_mask must be NULL when mask is NULL");
  DCN_CHECK(mask == nullptr || grad_mask != nullptr,
            "deform_conv2d_backward: grad_mask is required when mask is given");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const size_t x_bytes = (size_t)g.N * g.C * g.HW * sizeof(float);
  const size_t off_bytes = (size_t)g.N * 2 * g.dg * g.kk * g.P * sizeof(float);
  const size_t msk_bytes = (size_t)g.N * g.dg * g.kk * g.P * sizeof(float);
  const size_t w_bytes = (size_t)g.outC * g.Cg * g.kk * sizeof(float);
  auto dev_or_empty = [](const void* p, size_t bytes) { return bytes == 0 || is_device_ptr(p); };
  DCN_CHECK(dev_or_empty(grad_output, (size_t)g.N * g.outC * g.P) && dev_or_empty(input, x_bytes) &&
                dev_or_empty(weight, w_bytes) && dev_or_empty(offset, off_bytes),
            "deform_conv2d_backward: grad_output, input, weight and offset must be CUDA tensors");
  DCN_CHECK(dev_or_empty(grad_input, x_bytes) && dev_or_empty(grad_offset, off_bytes) &&
                dev_or_empty(grad_weight, w_bytes) &&
                (grad_mask == nullptr || dev_or_empty(grad_mask, msk_bytes)) &&
                (grad_bias == nullptr || dev_or_empty(grad_bias, (size_t)g.outC)),
            "deform_conv2d_backward: gradient outputs must be CUDA device buffers");
  DCN_CHECK(mask == nullptr || dev_or_empty(mask, msk_bytes), "mask must be a float32 CUDA tensor");

  const bool tc_bwd = use_tc_bwd(g, flags);
  const bool skip = g.N == 0 || g.C == 0 || g.outC == 0 || g.P == 0;  // .mm:779-782
  // the tensor-core prep kernel sums grad_bias while it reads grad_output
  const bool bias_in_prep = grad_bias != nullptr && tc_bwd && !skip;
  const bool no_pixels = (long long)g.N * g.P == 0;
  // Zero what the kernels accumulate into (.mm:764-777 zero-initialise too),
  // in one launch; the tensor-core path zeroes on its side streams instead.
  dcn::ZeroList z{};
  z.add(grad_offset, (long long)(off_bytes / sizeof(float)));
  z.add(grad_mask, (long long)(msk_bytes / sizeof(float)));
  const bool zero_on_side = tc_bwd && !skip;
  // (the tensor-core path adds grad_weight, or its tap-major workspace copy,
  // below)
  if (!zero_on_side) z.add(grad_weight, (long long)(w_bytes / sizeof(float)));
  if (no_pixels) z.add(grad_bias, g.outC);
  if (!zero_on_side) DCN_CUDA(dcn::launch_zero(z, stream), "zero");
  if (grad_bias != nullptr && !bias_in_prep && !no_pixels)
    DCN_CUDA(dcn::launch_grad_bias(grad_output, grad_bias, g, stream), "grad_bias");
  if (skip) {
    if (x_bytes) DCN_CUDA(cudaMemsetAsync(grad_input, 0, x_bytes, stream), "memset");
    return DCN_OK;
  }
  const size_t need = bwd_ws(g, flags);
  if (workspace_bytes < need || workspace == nullptr)
    return fail(DCN_ERR_WORKSPACE, "deform_conv2d_backward: workspace of %zu bytes needed, %zu given",
                need, workspace_bytes);
  Carver ws(align_ptr(workspace));
  // the caller's staging copy of the input (DCN_INPUT_STAGED), or our own
  const bool staged = flags & DCN_INPUT_STAGED;
  float* xt = staged ? const_cast<float*>(input) : ws.take(xt_floats(g));
  // the kernels accumulate grad_input in NHWC: into the caller's buffer when
  // it is channels-last, else into a workspace copy transposed at the end
  const bool nhwc = flags & DCN_INPUT_NHWC;
  // the accumulation uses 16-byte vector reductions
  DCN_CHECK(!nhwc || (reinterpret_cast<uintptr_t>(grad_input) & 15u) == 0,
            "deform_conv2d_backward: grad_input must be 16-byte aligned with DCN_INPUT_NHWC");
  float* gxt = nhwc ? grad_input : ws.take((size_t)g.N * g.HW * g.C);
  // xt (+ its zero row) and the zeroed grad-input accumulator in one pass;
  // with a staged input only the accumulator is zeroed
  auto stage_input = [&](cudaStream_t st) {
    if (staged) return cudaMemsetAsync(gxt, 0, x_bytes, st);
    return nhwc ? dcn::launch_copy_nhwc(input, xt, g.N, g.C, g.HW, true, gxt, st)
                : dcn::launch_nchw_to_nhwc(input, xt, g.N, g.C, g.HW, true, gxt, st);
  };
  const char* stage_name = staged ? "memset" : (nhwc ? "copy_nhwc" : "nchw_to_nhwc");
  if (tc_bwd) {
    const bool split = split_math(flags);
    const size_t parts = split ? 2 : 1;
    float* go_r = ws.take(parts * g.N * g.outC * ((g.P + 3) & ~3));
    float* wbt = ws.take(parts * g.outC * g.Cg * g.kk);
    const bool colp = use_col_path(g, flags);
    float* col = colp ? ws.take(dcn::tc_col_bytes(g, split) / sizeof(float)) : nullptr;
    // the weight gradient sums into a tap-major copy (coalesced reductions),
    // then puts it in grad_weight's layout
    float* gwt = ws.take(w_bytes / sizeof(float));
    z.add(gwt, (long long)(w_bytes / sizeof(float)));
    Fork fk(stream, side_streams_pay(g));  // one per call: it holds the side streams' lock
    // the fused kernel, then grad_input back to NCHW beside the grad_weight
    // layout (which sums grad_bias from the prologue's partial sums, if any)
    auto fused_rest = [&](const float* gpart, float* gb_out) -> int {
      DCN_CUDA(dcn::launch_bwd_fused_tc(g, go_r, wbt, xt, offset, mask, gxt, grad_offset,
                                        grad_mask, gwt, num_sms_current(), stream),
               "bwd_fused_tc");
      if (nhwc) {  // grad_input is complete: nothing to transpose
        DCN_CUDA(dcn::launch_weight_from_tap_major(gwt, grad_weight, g, stream, gpart, gb_out),
                 "grad_weight_layout");
        return DCN_OK;
      }
      if (dcn::bwd_finish_fits(gxt, grad_input, g)) {  // both in one launch
        DCN_CUDA(dcn::launch_bwd_finish(gxt, grad_input, gwt, grad_weight, g, gpart, gb_out,
                                        stream),
                 "bwd_finish");
        return DCN_OK;
      }
      DCN_ORDER(fk.fork(), "fork");
      DCN_CUDA_ON(fk.side(0),
                  dcn::launch_weight_from_tap_major(gwt, grad_weight, g, fk.side(0), gpart,
                                                    gb_out),
                  "grad_weight_layout");
      DCN_CUDA(dcn::launch_nhwc_to_nchw(gxt, grad_input, g.N, g.C, g.HW, stream), "nhwc_to_nchw");
      DCN_ORDER(fk.join(0), "join");
      return DCN_OK;
    };
    if (staged && use_fused_bwd(g, flags)) {
      // the helpers in one launch on the caller's stream (no cross-stream
      // waits): grad_out rows with grad_bias partial sums, the packed weight,
      // the zeroed accumulators
      float* gpart = ws.take(dcn::tc_bias_part_floats(g));
      z.add(gxt, (long long)(x_bytes / sizeof(float)));
      DCN_CUDA(dcn::launch_bwd_prologue(g, grad_output, go_r, bias_in_prep ? gpart : nullptr,
                                        weight, wbt, z, stream),
               "bwd_prologue");
      return fused_rest(gpart, bias_in_prep ? grad_bias : nullptr);
    }
    // The grad_out prep (after zeroing grad_bias, which it sums into) stays
    // on the caller's stream, where it starts at once: it is the longest
    // helper.  The weight pack + the zeroing of the other accumulators (side
    // 0) and the input staging or the grad-input zeroing (side 1) run beside
    // it, behind the cross-stream wait.
    DCN_ORDER(fk.fork(), "fork");
    DCN_CUDA_ON(fk.side(0), dcn::launch_tc_pack_weight_bwd(weight, wbt, g, split, fk.side(0)),
                "tc_pack_weight_bwd");
    DCN_CUDA_ON(fk.side(0), dcn::launch_zero(z, fk.side(0)), "zero");
    DCN_CUDA_ON(fk.side(1), stage_input(fk.side(1)), stage_name);
    if (bias_in_prep)
      DCN_CUDA(cudaMemsetAsync(grad_bias, 0, (size_t)g.outC * sizeof(float), stream), "memset");
    DCN_CUDA(dcn::launch_tc_prep_go(g, grad_output, go_r, bias_in_prep ? grad_bias : nullptr,
                                    split, stream),
             "tc_prep_go");
    DCN_ORDER(fk.join(0), "join");
    DCN_ORDER(fk.join(1), "join");
    if (use_fused_bwd(g, flags)) return fused_rest(nullptr, nullptr);
    DCN_CUDA(dcn::launch_bwd_data_tc(g, go_r, split, wbt, xt, offset, mask, gxt, grad_offset,
                                     grad_mask, col, stream),
             "bwd_data_tc");
    if (nhwc) {  // grad_input is complete: nothing to transpose
      if (colp) {
        DCN_CUDA(dcn::launch_bwd_weight_col(g, col, go_r, gwt, true, split, num_sms_current(),
                                            stream),
                 "bwd_weight_col");
      } else {
        void* plans = ws.take(dcn::tc_plan_bytes(g) / sizeof(float));
        DCN_CUDA(dcn::launch_tc_plans(g, offset, mask, plans, stream), "tc_plans");
        DCN_CUDA(dcn::launch_bwd_weight_tc(g, go_r, xt, plans, gwt, true, split,
                                           num_sms_current(), stream),
                 "bwd_weight_tc");
      }
      DCN_CUDA(dcn::launch_weight_from_tap_major(gwt, grad_weight, g, stream),
               "grad_weight_layout");
      return DCN_OK;
    }
    // grad_input back to NCHW (side 0) beside the weight gradient
    DCN_ORDER(fk.fork(), "fork");
    DCN_CUDA_ON(fk.side(0), dcn::launch_nhwc_to_nchw(gxt, grad_input, g.N, g.C, g.HW, fk.side(0)),
                "nhwc_to_nchw");
    if (colp) {
      DCN_CUDA(dcn::launch_bwd_weight_col(g, col, go_r, gwt, true, split, num_sms_current(),
                                          stream),
               "bwd_weight_col");
    } else {
      void* plans = ws.take(dcn::tc_plan_bytes(g) / sizeof(float));
      DCN_CUDA(dcn::launch_tc_plans(g, offset, mask, plans, stream), "tc_plans");
      DCN_CUDA(dcn::launch_bwd_weight_tc(g, go_r, xt, plans, gwt, true, split,
                                         num_sms_current(), stream),
               "bwd_weight_tc");
    }
    DCN_CUDA(dcn::launch_weight_from_tap_major(gwt, grad_weight, g, stream),
             "grad_weight_layout");
    DCN_ORDER(fk.join(0), "join");
    return DCN_OK;
  }
  DCN_CUDA(stage_input(stream), stage_name);
  if (dcn::dgroup_supported(g) && !(flags & (DCN_ALGO_SIMT_GEMM | DCN_ALGO_SIMT_DIRECT))) {
    DCN_CUDA(dcn::launch_bwd_dgroup(g, grad_output, weight, xt, offset, mask, gxt, grad_offset,
                                    grad_mask, grad_weight, stream),
             "bwd_dgroup");
    if (!nhwc)
      DCN_CUDA(dcn::launch_nhwc_to_nchw(gxt, grad_input, g.N, g.C, g.HW, stream), "nhwc_to_nchw");
    return DCN_OK;
  }
  if (dcn::bwd_small_supported(g) && !(flags & DCN_ALGO_SIMT_GEMM)) {
    DCN_CUDA(dcn::launch_bwd_small(g, grad_output, weight, xt, offset, mask, gxt, grad_offset,
                                   grad_mask, grad_weight, stream),
             "bwd_small");
    if (!nhwc)
      DCN_CUDA(dcn::launch_nhwc_to_nchw(gxt, grad_input, g.N, g.C, g.HW, stream), "nhwc_to_nchw");
    return DCN_OK;
  }
  float* wb = ws.take((size_t)g.G * g.kk * g.Og * g.Cg);
  DCN_CUDA(dcn::launch_pack_weight_bwd(weight, wb, g, stream), "pack_weight_bwd");
  DCN_CUDA(dcn::launch_bwd_data_simt(g, grad_output, wb, xt, offset, mask, gxt, grad_offset,
                                     grad_mask, stream),
           "bwd_data_simt");
  if (!nhwc)
    DCN_CUDA(dcn::launch_nhwc_to_nchw(gxt, grad_input, g.N, g.C, g.HW, stream), "nhwc_to_nchw");
  DCN_CUDA(dcn::launch_bwd_weight_simt(g, grad_output, xt, offset, mask, grad_weight,
                                       num_sms_current(), stream),
           "bwd_weight_simt");
  return DCN_OK;
}

DCN_API int dcn_forward(const dcn_shape* s, const float* input, const float* weight,
                        const float* offset, const float* mask, const float* bias,
                        float* output, uint32_t flags, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return forward_core(s, 0, -1, input, weight, offset, mask, bias, output, flags, workspace,
                      workspace_bytes, stream);
}

DCN_API int dcn_forward_rows(const dcn_shape* s, int64_t row_begin, int64_t rows,
                             const float* input, const float* weight, const float* offset,
                             const float* mask, const float* bias, float* output, uint32_t flags,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (rows <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "deform_conv2d_forward: rows must be positive");
  return forward_core(s, row_begin, rows, input, weight, offset, mask, bias, output, flags,
                      workspace, workspace_bytes, stream);
}

DCN_API int dcn_backward(const dcn_shape* s, const float* grad_output, const float* input,
                         const float* weight, const float* offset, const float* mask,
                         float* grad_input, float* grad_offset, float* grad_mask,
                         float* grad_weight, float* grad_bias, uint32_t flags,
                         void* workspace, size_t workspace_bytes, void* stream) {
  return backward_core(s, 0, -1, grad_output, input, weight, offset, mask, grad_input,
                       grad_offset, grad_mask, grad_weight, grad_bias, flags, workspace,
                       workspace_bytes, stream);
}

DCN_API int dcn_backward_rows(const dcn_shape* s, int64_t row_begin, int64_t rows,
                              const float* grad_output, const float* input, const float* weight,
                              const float* offset, const float* mask, float* grad_input,
                              float* grad_offset, float* grad_mask, float* grad_weight,
                              float* grad_bias, uint32_t flags, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (rows <= 0)
    return fail(DCN_ERR_INVALID_ARGUMENT, "deform_conv2d_backward: rows must be positive");
  return backward_core(s, row_begin, rows, grad_output, input, weight, offset, mask, grad_input,
                       grad_offset, grad_mask, grad_weight, grad_bias, flags, workspace,
                       workspace_bytes, stream);
}

// fp32 copies for the 16-bit backward: grad_output, input, weight, offset,
// mask, and the five gradients (input, offset, mask, weight, bias).
static size_t bwd_bf16_copy_bytes(const dcn::Geom& g) {
  const size_t x = align_up((size_t)g.N * g.C * g.HW * 4), w = align_up((size_t)g.outC * g.Cg * g.kk * 4);
  const size_t off = align_up((size_t)g.N * 2 * g.dg * g.kk * g.P * 4);
  const size_t m = align_up((size_t)g.N * g.dg * g.kk * g.P * 4);
  const size_t go = align_up((size_t)g.N * g.outC * g.P * 4), b = align_up((size_t)g.outC * 4);
  return go + 2 * (x + w + off + m) + b;
}

// The fused 16-bit tensor-core backward (kind::f16 operands of the tensors'
// type) where it covers the shape and no other kernel family is pinned.
static bool use_fused16(const dcn::Geom& g, uint32_t flags) {
  return !(flags & (DCN_ALGO_SIMT_GEMM | DCN_ALGO_SIMT_DIRECT | DCN_ALGO_TC_GATHER_WEIGHT |
                    DCN_ALGO_TC_COLUMN_BUFFER)) &&
         g.N > 0 && g.C > 0 && g.outC > 0 && g.P > 0 && dcn::tc_fused16_supported(g);
}

// Its workspace: the 16-bit staging copy, grad_out rows and packed weight;
// fp32 accumulators of grad_input (NHWC), grad_offset, grad_mask, the
// tap-major grad_weight and grad_bias.
static size_t bwd_fused16_bytes(const dcn::Geom& g, bool staged) {
  const size_t w = (size_t)g.outC * g.Cg * g.kk;
  return (staged ? 0 : align_up(((size_t)g.N * g.HW * g.C + g.C) * 2)) +
         align_up((size_t)g.N * g.outC * ((g.P + 7) & ~7) * 2) + align_up(w * 2) +
         align_up((size_t)g.N * g.HW * g.C * 4) + align_up((size_t)g.N * 2 * g.dg * g.kk * g.P * 4) +
         align_up((size_t)g.N * g.dg * g.kk * g.P * 4) + align_up(w * 4) +
         align_up(dcn::tc_bias_part_floats16(g) * 4) + kAlign;
}

static size_t bwd_h16_ws(const dcn::Geom& g, uint32_t flags) {
  return use_fused16(g, flags)
             ? bwd_fused16_bytes(g, flags & DCN_INPUT_STAGED)
             : bwd_bf16_copy_bytes(g) + kAlign + bwd_ws(g, flags & ~(uint32_t)DCN_INPUT_STAGED);
}

DCN_API size_t dcn_backward_bf16_workspace_size(const dcn_shape* s, uint32_t flags) {
  dcn::Geom g;
  if (make_geom(s, true, true, g, "dcn_backward_bf16_workspace_size") != DCN_OK) return 0;
  return bwd_h16_ws(g, flags);
}

// The 16-bit backward (bf16, or fp16 with `f16`): the fp32 backward on upcast
// copies, the gradients rounded back.
static int backward_h16(bool f16, const dcn_shape* s, const void* grad_output, const void* input,
                        const void* weight, const void* offset, const void* mask,
                        void* grad_input, void* grad_offset, void* grad_mask, void* grad_weight,
                        void* grad_bias, uint32_t flags, void* workspace,
                        size_t workspace_bytes, void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = make_geom(s, mask != nullptr, grad_bias != nullptr, g, "deform_conv2d_backward");
  if (rc != DCN_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const bool staged = flags & DCN_INPUT_STAGED;
  if (use_fused16(g, flags)) {
    DCN_CHECK(mask != nullptr || grad_mask == nullptr,
              "deform_conv2d_backward: grad_mask must be NULL when mask is NULL");
    DCN_CHECK(mask == nullptr || grad_mask != nullptr,
              "deform_conv2d_backward: grad_mask is required when mask is given");
    g.mask_logits = (flags & DCN_MASK_LOGITS) && mask != nullptr ? 1 : 0;
    apply_test_flags(g, flags);
    DCN_CHECK(is_device_ptr(grad_output) && is_device_ptr(input) && is_device_ptr(weight) &&
                  is_device_ptr(offset) && (mask == nullptr || is_device_ptr(mask)),
              "deform_conv2d_backward: grad_output, input, weight and offset must be CUDA tensors");
    DCN_CHECK(is_device_ptr(grad_input) && is_device_ptr(grad_offset) &&
                  is_device_ptr(grad_weight) && (grad_mask == nullptr || is_device_ptr(grad_mask)) &&
                  (grad_bias == nullptr || is_device_ptr(grad_bias)),
              "deform_conv2d_backward: gradient outputs must be CUDA device buffers");
    const size_t need16 = bwd_fused16_bytes(g, staged);
    if (workspace_bytes < need16 || workspace == nullptr)
      return fail(DCN_ERR_WORKSPACE,
                  "deform_conv2d_backward: workspace of %zu bytes needed, %zu given", need16,
                  workspace_bytes);
    char* p = static_cast<char*>(align_ptr(workspace));
    auto take = [&p](size_t bytes) {
      char* q = p;
      p += align_up(bytes);
      return q;
    };
    const long long nx = (long long)g.N * g.HW * g.C, nw = (long long)g.outC * g.Cg * g.kk;
    const long long noff = (long long)g.N * 2 * g.dg * g.kk * g.P;
    const long long nm = (long long)g.N * g.dg * g.kk * g.P;
    // the caller's 16-bit staging copy (DCN_INPUT_STAGED), or our own
    void* xt = staged ? const_cast<void*>(input) : take(((size_t)nx + g.C) * 2);
    void* go_r = take((size_t)g.N * g.outC * ((g.P + 7) & ~7) * 2);
    void* wbt = take((size_t)nw * 2);
    float* gxt = reinterpret_cast<float*>(take((size_t)nx * 4));
    float* goff = reinterpret_cast<float*>(take((size_t)noff * 4));
    float* gm = reinterpret_cast<float*>(take((size_t)nm * 4));
    float* gwt = reinterpret_cast<float*>(take((size_t)nw * 4));
    float* gpart = reinterpret_cast<float*>(take(dcn::tc_bias_part_floats16(g) * 4));
    const bool nhwc = flags & DCN_INPUT_NHWC;
    dcn::ZeroList z{};
    z.add(goff, noff);
    if (mask) z.add(gm, nm);
    z.add(gwt, nw);
    z.add(gxt, nx);
    // the input staging (unless staged) on a side stream beside the helpers'
    // one launch: grad_out rows with grad_bias partial sums, the packed
    // weight, the zeroed accumulators
    Fork fk(stream, side_streams_pay(g));  // one per call: it holds the side streams' lock
    if (!staged) {
      DCN_ORDER(fk.fork(), "fork");
      const cudaStream_t s1 = fk.side(1);
      if (nhwc) {  // channels-last: a copy plus the zero row
        DCN_CUDA_ON(s1,
                    cudaMemcpyAsync(xt, input, (size_t)nx * 2, cudaMemcpyDeviceToDevice, s1),
                    "copy");
        DCN_CUDA_ON(s1,
                    cudaMemsetAsync(static_cast<char*>(xt) + (size_t)nx * 2, 0,
                                    (size_t)g.C * 2, s1),
                    "memset");
      } else {
        DCN_CUDA_ON(s1,
                    dcn::launch_nchw_to_nhwc_bf16(input, xt, g.N, g.C, g.HW, /*zero_row=*/true,
                                                  s1),
                    "nchw_to_nhwc");
      }
    }
    DCN_CUDA(dcn::launch_bwd_prologue16(g, grad_output, go_r, grad_bias ? gpart : nullptr,
                                        weight, wbt, z, f16, stream),
             "bwd_prologue");
    if (!staged) DCN_ORDER(fk.join(1), "join");
    DCN_CUDA(dcn::launch_bwd_fused_tc_h16(g, go_r, wbt, xt, offset, mask, gxt, goff,
                                          mask ? gm : nullptr, gwt, f16, num_sms_current(),
                                          stream),
             f16 ? "bwd_fused_tc_f16" : "bwd_fused_tc_bf16");
    // grad_input back to the tensors' layout and type, the other gradients
    // rounded (grad_bias summed from its parts) beside it (side 0)
    dcn::H16List rest{};
    rest.add(goff, grad_offset, noff);
    if (mask) rest.add(gm, grad_mask, nm);
    DCN_ORDER(fk.fork(), "fork");
    DCN_CUDA_ON(fk.side(0),
                dcn::launch_grads_to_h16(gwt, grad_weight, g, rest, f16, fk.side(0), gpart,
                                         grad_bias),
                "grads_to_h16");
    if (nhwc)
      DCN_CUDA(dcn::launch_f32_to_h16(gxt, grad_input, nx, f16, stream),
               f16 ? "f32_to_f16" : "f32_to_bf16");
    else
      DCN_CUDA(dcn::launch_nhwc_to_nchw16(gxt, grad_input, g.N, g.C, g.HW, f16, stream),
               "nhwc_to_nchw");
    DCN_ORDER(fk.join(0), "join");
    return DCN_OK;
  }
  DCN_CHECK(!staged, "deform_conv2d_backward: a 16-bit staging copy needs the tensor-core "
                     "backward, which does not cover this shape");
  const size_t need = bwd_bf16_copy_bytes(g) + kAlign + bwd_ws(g, flags);
  if (workspace_bytes < need || workspace == nullptr)
    return fail(DCN_ERR_WORKSPACE, "deform_conv2d_backward: workspace of %zu bytes needed, %zu given",
                need, workspace_bytes);
  char* base = static_cast<char*>(align_ptr(workspace));
  Carver ws(base);
  const long long nx = (long long)g.N * g.C * g.HW, nw = (long long)g.outC * g.Cg * g.kk;
  const long long noff = (long long)g.N * 2 * g.dg * g.kk * g.P;
  const long long nm = (long long)g.N * g.dg * g.kk * g.P, ngo = (long long)g.N * g.outC * g.P;
  float* go32 = ws.take(ngo);
  float* x32 = ws.take(nx);
  float* w32 = ws.take(nw);
  float* off32 = ws.take(noff);
  float* m32 = ws.take(nm);
  float* gx32 = ws.take(nx);
  float* gw32 = ws.take(nw);
  float* goff32 = ws.take(noff);
  float* gm32 = ws.take(nm);
  float* gb32 = ws.take(g.outC);
  const char* up = f16 ? "f16_to_f32" : "bf16_to_f32";
  const char* down = f16 ? "f32_to_f16" : "f32_to_bf16";
  DCN_CUDA(dcn::launch_h16_to_f32(grad_output, go32, ngo, f16, stream), up);
  DCN_CUDA(dcn::launch_h16_to_f32(input, x32, nx, f16, stream), up);
  DCN_CUDA(dcn::launch_h16_to_f32(weight, w32, nw, f16, stream), up);
  DCN_CUDA(dcn::launch_h16_to_f32(offset, off32, noff, f16, stream), up);
  if (mask) DCN_CUDA(dcn::launch_h16_to_f32(mask, m32, nm, f16, stream), up);
  const size_t used = bwd_bf16_copy_bytes(g);
  rc = dcn_backward(s, go32, x32, w32, off32, mask ? m32 : nullptr, gx32, goff32,
                    mask ? gm32 : nullptr, gw32, grad_bias ? gb32 : nullptr, flags, base + used,
                    workspace_bytes - (size_t)(base - static_cast<char*>(workspace)) - used,
                    stream_);
  if (rc != DCN_OK) return rc;
  DCN_CUDA(dcn::launch_f32_to_h16(gx32, grad_input, nx, f16, stream), down);
  DCN_CUDA(dcn::launch_f32_to_h16(goff32, grad_offset, noff, f16, stream), down);
  if (mask) DCN_CUDA(dcn::launch_f32_to_h16(gm32, grad_mask, nm, f16, stream), down);
  DCN_CUDA(dcn::launch_f32_to_h16(gw32, grad_weight, nw, f16, stream), down);
  if (grad_bias) DCN_CUDA(dcn::launch_f32_to_h16(gb32, grad_bias, g.outC, f16, stream), down);
  return DCN_OK;
}

DCN_API int dcn_backward_bf16(const dcn_shape* s, const void* grad_output, const void* input,
                              const void* weight, const void* offset, const void* mask,
                              void* grad_input, void* grad_offset, void* grad_mask,
                              void* grad_weight, void* grad_bias, uint32_t flags,
                              void* workspace, size_t workspace_bytes, void* stream) {
  return backward_h16(false, s, grad_output, input, weight, offset, mask, grad_input, grad_offset,
                      grad_mask, grad_weight, grad_bias, flags, workspace, workspace_bytes,
                      stream);
}

DCN_API size_t dcn_backward_f16_workspace_size(const dcn_shape* s, uint32_t flags) {
  dcn::Geom g;
  if (make_geom(s, true, true, g, "dcn_backward_f16_workspace_size") != DCN_OK) return 0;
  return bwd_h16_ws(g, flags);
}

DCN_API int dcn_backward_f16(const dcn_shape* s, const void* grad_output, const void* input,
                             const void* weight, const void* offset, const void* mask,
                             void* grad_input, void* grad_offset, void* grad_mask,
                             void* grad_weight, void* grad_bias, uint32_t flags, void* workspace,
                             size_t workspace_bytes, void* stream) {
  return backward_h16(true, s, grad_output, input, weight, offset, mask, grad_input, grad_offset,
                      grad_mask, grad_weight, grad_bias, flags, workspace, workspace_bytes,
                      stream);
}

static int single_geom(dcn::Geom& g, int64_t C, int64_t H, int64_t W, int64_t kh, int64_t kw,
                       int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                       int64_t dg, bool use_mask, const char* op) {
  dcn_shape s;
  s.batch = 1; s.in_channels = C; s.height = H; s.width = W; s.out_channels = C;
  s.kernel_h = kh; s.kernel_w = kw; s.stride_h = sh; s.stride_w = sw; s.pad_h = ph; s.pad_w = pw;
  s.dilation_h = dh; s.dilation_w = dw; s.groups = 1; s.deformable_groups = dg;
  return make_geom(&s, use_mask, false, g, op);
}

DCN_API int dcn_col2im(const float* columns, const float* offset, const float* mask,
                       float* grad_im, int64_t C, int64_t H, int64_t W, int64_t kh, int64_t kw,
                       int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                       int64_t dg, void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = single_geom(g, C, H, W, kh, kw, sh, sw, ph, pw, dh, dw, dg, mask != nullptr,
                       "deformable_col2im");
  if (rc != DCN_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const size_t im_bytes = (size_t)C * H * W * sizeof(float);
  if (im_bytes == 0) return DCN_OK;
  DCN_CHECK(is_device_ptr(grad_im), "deformable_col2im: grad_im must be a CUDA device buffer");
  DCN_CUDA(cudaMemsetAsync(grad_im, 0, im_bytes, stream), "memset");
  if ((long long)C * g.kk * g.P == 0) return DCN_OK;
  DCN_CHECK(is_device_ptr(columns) && is_device_ptr(offset),
            "deformable_col2im: columns and offset must be CUDA tensors");
  DCN_CHECK(mask == nullptr || is_device_ptr(mask), "mask must be a float32 CUDA tensor");
  DCN_CUDA(dcn::launch_col2im_single(g, columns, offset, mask, grad_im, stream), "col2im");
  return DCN_OK;
}

DCN_API int dcn_col2im_coord(const float* columns, const float* input, const float* offset,
                             const float* mask, float* grad_offset, float* grad_mask, int64_t C,
                             int64_t H, int64_t W, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                             int64_t ph, int64_t pw, int64_t dh, int64_t dw, int64_t dg,
                             void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = single_geom(g, C, H, W, kh, kw, sh, sw, ph, pw, dh, dw, dg, mask != nullptr,
                       "deformable_col2im_coord");
  if (rc != DCN_OK) return rc;
  DCN_CHECK(mask != nullptr || grad_mask == nullptr,
            "deformable_col2im_coord: grad_mask must be NULL when mask is NULL");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const long long total = 2LL * g.dg * g.kk * g.P;
  if (total == 0) return DCN_OK;
  DCN_CHECK(is_device_ptr(grad_offset) && (mask == nullptr || is_device_ptr(grad_mask)),
            "deformable_col2im_coord: gradient outputs must be CUDA device buffers");
  DCN_CHECK(is_device_ptr(offset) && (C == 0 || (is_device_ptr(columns) && is_device_ptr(input))),
            "deformable_col2im_coord: columns, input and offset must be CUDA tensors");
  DCN_CHECK(mask == nullptr || is_device_ptr(mask), "mask must be a float32 CUDA tensor");
  DCN_CUDA(dcn::launch_col2im_coord_single(g, columns, input, offset, mask, grad_offset, grad_mask,
                                           stream),
           "col2im_coord");
  return DCN_OK;
}

DCN_API size_t dcn_staged_input_size(const dcn_shape* s) {
  dcn::Geom g;
  if (make_geom(s, false, false, g, "dcn_staged_input_size") != DCN_OK) return 0;
  return xt_floats(g) * sizeof(float);
}

DCN_API int dcn_stage_input(const dcn_shape* s, const float* input, float* staged,
                            uint32_t flags, void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = make_geom(s, false, false, g, "dcn_stage_input");
  if (rc != DCN_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DCN_CHECK(is_device_ptr(staged), "dcn_stage_input: staged must be a CUDA device buffer");
  DCN_CHECK((long long)g.N * g.C * g.HW == 0 || is_device_ptr(input),
            "dcn_stage_input: input must be a CUDA tensor");
  if (flags & DCN_INPUT_NHWC)
    DCN_CUDA(dcn::launch_copy_nhwc(input, staged, g.N, g.C, g.HW, true, nullptr, stream),
             "copy_nhwc");
  else
    DCN_CUDA(dcn::launch_nchw_to_nhwc(input, staged, g.N, g.C, g.HW, true, nullptr, stream),
             "nchw_to_nhwc");
  return DCN_OK;
}

DCN_API size_t dcn_staged_input_size_h16(const dcn_shape* s) {
  dcn::Geom g;
  if (make_geom(s, false, false, g, "dcn_staged_input_size_h16") != DCN_OK) return 0;
  return ((size_t)g.N * g.HW * g.C + g.C) * 2;
}

DCN_API int dcn_stage_input_h16(const dcn_shape* s, const void* input, void* staged,
                                uint32_t flags, void* stream_) {
  g_last_error.clear();
  dcn::Geom g;
  int rc = make_geom(s, false, false, g, "dcn_stage_input_h16");
  if (rc != DCN_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const size_t nx = (size_t)g.N * g.HW * g.C;
  DCN_CHECK(is_device_ptr(staged), "dcn_stage_input_h16: staged must be a CUDA device buffer");
  DCN_CHECK(nx == 0 || is_device_ptr(input), "dcn_stage_input_h16: input must be a CUDA tensor");
  if (flags & DCN_INPUT_NHWC) {  // a copy plus the zero row
    if (nx) DCN_CUDA(cudaMemcpyAsync(staged, input, nx * 2, cudaMemcpyDeviceToDevice, stream), "copy");
    DCN_CUDA(cudaMemsetAsync(static_cast<char*>(staged) + nx * 2, 0, (size_t)g.C * 2, stream),
             "memset");
  } else {
    DCN_CUDA(dcn::launch_nchw_to_nhwc_bf16(input, staged, g.N, g.C, g.HW, /*zero_row=*/true,
                                           stream),
             "nchw_to_nhwc");
  }
  return DCN_OK;
}

DCN_API int dcn_h16_staging(const dcn_shape* s, uint32_t flags) {
  dcn::Geom g;
  if (make_geom(s, true, true, g, "dcn_h16_staging") != DCN_OK) return 0;
  return use_bf16_tc(g, flags) && use_fused16(g, flags) ? 1 : 0;
}

DCN_API int dcn_device_status(void* stream_, int clear, int* status) {
  g_last_error.clear();
  DCN_CHECK(status != nullptr, "dcn_device_status: status must not be NULL");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int f = 0, b = 0;
  cudaError_t e = dcn::read_fwd_status(&f, clear != 0, stream);
  if (e == cudaSuccess) e = dcn::read_bwd_status(&b, clear != 0, stream);
  if (e != cudaSuccess) return cuda_fail(e, "dcn_device_status");
  *status = f | b;
  return DCN_OK;
}

DCN_API int dcn_profiler_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_on = enable != 0;
  return DCN_OK;
}

DCN_API int dcn_profiler_read(dcn_kernel_stat* stats, int max_stats, int* count) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  std::map<std::string, std::pair<int64_t, double>> agg;
  std::vector<std::string> order;
  int rc = DCN_OK;
  for (auto& r : g_prof_recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.stop) != cudaSuccess ||
        cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) {
      cudaGetLastError();
      rc = fail(DCN_ERR_CUDA, "dcn_profiler_read: event query failed");
    }
    if (!agg.count(r.name)) order.push_back(r.name);
    auto& a = agg[r.name];
    a.first += 1;
    a.second += ms;
    g_prof_pool.push_back(r.start);
    g_prof_pool.push_back(r.stop);
  }
  g_prof_recs.clear();
  int n = 0;
  for (auto& name : order) {
    if (stats && n < max_stats) {
      std::memset(&stats[n], 0, sizeof(dcn_kernel_stat));
      std::strncpy(stats[n].name, name.c_str(), sizeof(stats[n].name) - 1);
      stats[n].launches = agg[name].first;
      stats[n].total_ms = agg[name].second;
    }
    ++n;
  }
  if (count) *count = n;
  return rc;
}

}  // extern "C"
