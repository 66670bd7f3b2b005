// The C ABI of libsdxcuda (include/sdxcuda.h): runtime, weight packing, op entry points and the
// graph-captured session. No C++ exception crosses this boundary; errors are status codes plus a
// thread-local message.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "../../include/sdxcuda.h"
#include "sdx_internal.h"

namespace sdx {

static thread_local char t_msg[512] = "";
static std::atomic<uint64_t> g_launches{0};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(cudaError_t e, const char* what) {
  snprintf(t_msg, sizeof(t_msg), "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
  return e == cudaErrorMemoryAllocation ? SDX_ERR_OOM : SDX_ERR_CUDA;
}

void clear_error() { t_msg[0] = 0; }

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

PFN_encodeTiled get_encode_tiled() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

int num_sms(int device) {
  static std::atomic<int> cache[SDX_MAX_DEVICES];
  const bool slot = device >= 0 && device < SDX_MAX_DEVICES;
  if (slot) {
    const int c = cache[device].load(std::memory_order_relaxed);
    if (c) return c;
  }
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  if (slot) cache[device].store(n, std::memory_order_relaxed);
  return n;
}

int raise_smem_limit(SmemAttr& rec, const void* fn, int bytes, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, what);
  if (dev < 0 || dev >= SDX_MAX_DEVICES) return set_error(SDX_ERR_INVALID, "%s: device ordinal %d out of range", what, dev);
  if (rec.bytes[dev].load(std::memory_order_acquire) >= bytes) return SDX_OK;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return set_cuda_error(e, what);
  int cur = rec.bytes[dev].load(std::memory_order_relaxed);
  while (cur < bytes && !rec.bytes[dev].compare_exchange_weak(cur, bytes, std::memory_order_release)) {
  }
  return SDX_OK;
}

// ---- host-side fault injection (tests only; never touches the GPU)
static std::mutex g_fault_mu;
static int g_fault_kind = 0, g_fault_nth = 0, g_fault_seen = 0;

bool inject_fire(int kind) {
  std::lock_guard<std::mutex> lk(g_fault_mu);
  if (g_fault_kind != kind || g_fault_nth <= 0) return false;
  if (++g_fault_seen == g_fault_nth) {
    g_fault_kind = 0;
    g_fault_nth = 0;
    return true;
  }
  return false;
}

}  // namespace sdx

using namespace sdx;

#define CK(call, what)                                   \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return set_cuda_error(e_, what); \
  } while (0)

static inline cudaStream_t S(sdx_ctx* ctx, sdx_stream s) {
  return s ? static_cast<cudaStream_t>(s) : ctx->stream;
}

static int use_ctx(sdx_ctx* ctx) {
  if (!ctx) return set_error(SDX_ERR_INVALID, "null context");
  if (ctx->poisoned) return set_error(SDX_ERR_POISONED, "context saw a device error; close and reopen it");
  CK(cudaSetDevice(ctx->device), "cudaSetDevice");
  return SDX_OK;
}

#define USE(ctx)                 \
  do {                           \
    int rc_ = use_ctx(ctx);      \
    if (rc_) return rc_;         \
  } while (0)

#define LAUNCH_GUARD()                                                                       \
  do {                                                                                       \
    if (inject_fire(FAULT_LAUNCH)) return set_error(SDX_ERR_INJECTED, "injected launch fault"); \
  } while (0)

template <typename T>
static inline T* P(sdx_dptr p) {
  return reinterpret_cast<T*>(p);
}

// Channel-sum scratch of sdx_channel_gate_static. It is a fixed file-scope device array (the
// runtime places one copy on each device when the module loads), so that entry point never
// allocates. Every entry a call reads is first written by the same call, so nothing has to be
// cleared between calls; the array simply keeps the partial sums of the last call.
static __device__ __align__(256) float g_gate_static_partial[SDX_GATE_STATIC_MAX_SCRATCH_BYTES / sizeof(float)];

// Device address of g_gate_static_partial on `device` (the current device), looked up on the
// first call for that device and cached. The address stays valid while the device's primary
// context lives.
static int gate_static_scratch(int device, float** out) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static float* cached[kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices) return set_error(SDX_ERR_INVALID, "channel gate (static): device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[device]) {
    void* p = nullptr;
    CK(cudaGetSymbolAddress(&p, g_gate_static_partial), "cudaGetSymbolAddress(channel gate scratch)");
    if (!p) return set_error(SDX_ERR_CUDA, "channel gate (static): scratch array has no device address");
    cached[device] = static_cast<float*>(p);
  }
  *out = cached[device];
  return SDX_OK;
}

extern "C" {

int sdx_abi_version(void) { return SDX_ABI_VERSION; }

int sdx_last_error(char* buf, int len) {
  if (!buf || len <= 0) return SDX_ERR_INVALID;
  snprintf(buf, (size_t)len, "%s", t_msg);
  return SDX_OK;
}

int sdx_device_count(int* count) {
  if (!count) return set_error(SDX_ERR_INVALID, "null count");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *count = 0;
    return SDX_OK;
  }
  *count = n;
  return SDX_OK;
}

int sdx_open(int ordinal, sdx_ctx** out) {
  if (!out) return set_error(SDX_ERR_INVALID, "null out");
  int n = 0;
  sdx_device_count(&n);
  if (ordinal < 0 || ordinal >= n) return set_error(SDX_ERR_INVALID, "device %d not present (%d devices)", ordinal, n);
  CK(cudaSetDevice(ordinal), "cudaSetDevice");
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, ordinal), "cudaGetDeviceProperties");
  if (prop.major != 10) return set_error(SDX_ERR_NOT_SUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", ordinal, prop.major, prop.minor);
  sdx_ctx* c = new (std::nothrow) sdx_ctx();
  if (!c) return set_error(SDX_ERR_OOM, "context allocation");
  c->device = ordinal;
  c->poisoned = 0;
  c->sm_count = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return set_cuda_error(e, "cudaStreamCreate");
  }
  e = cudaMalloc(&c->err_word, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(c->err_word, 0, sizeof(unsigned int));
  if (e != cudaSuccess) {
    cudaStreamDestroy(c->stream);
    delete c;
    return set_cuda_error(e, "error word");
  }
  *out = c;
  return SDX_OK;
}

int sdx_close(sdx_ctx* ctx) {
  if (!ctx) return SDX_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->err_word);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return SDX_OK;
}

int sdx_ctx_stream(sdx_ctx* ctx, sdx_stream* stream) {
  if (!ctx || !stream) return set_error(SDX_ERR_INVALID, "null argument");
  *stream = ctx->stream;
  return SDX_OK;
}

int sdx_device_info(sdx_ctx* ctx, char* name, int name_len, int* sm_count, int* cc_major, int* cc_minor,
                    size_t* total_mem) {
  if (!ctx) return set_error(SDX_ERR_INVALID, "null context");
  cudaDeviceProp p;
  CK(cudaGetDeviceProperties(&p, ctx->device), "cudaGetDeviceProperties");
  if (name && name_len > 0) snprintf(name, (size_t)name_len, "%s", p.name);
  if (sm_count) *sm_count = p.multiProcessorCount;
  if (cc_major) *cc_major = p.major;
  if (cc_minor) *cc_minor = p.minor;
  if (total_mem) *total_mem = p.totalGlobalMem;
  return SDX_OK;
}

int sdx_malloc(sdx_ctx* ctx, size_t bytes, sdx_dptr* out) {
  USE(ctx);
  if (!out) return set_error(SDX_ERR_INVALID, "null out");
  if (inject_fire(FAULT_MALLOC)) return set_error(SDX_ERR_INJECTED, "injected allocation fault");
  void* p = nullptr;
  CK(cudaMalloc(&p, std::max<size_t>(bytes, 256)), "cudaMalloc");
  *out = reinterpret_cast<sdx_dptr>(p);
  return SDX_OK;
}

int sdx_free(sdx_ctx* ctx, sdx_dptr p) {
  if (!ctx) return set_error(SDX_ERR_INVALID, "null context");
  cudaSetDevice(ctx->device);
  if (p) CK(cudaFree(reinterpret_cast<void*>(p)), "cudaFree");
  return SDX_OK;
}

int sdx_host_alloc_pinned(size_t bytes, void** out) {
  if (!out) return set_error(SDX_ERR_INVALID, "null out");
  if (inject_fire(FAULT_MALLOC)) return set_error(SDX_ERR_INJECTED, "injected allocation fault");
  CK(cudaHostAlloc(out, std::max<size_t>(bytes, 64), cudaHostAllocPortable), "cudaHostAlloc");
  return SDX_OK;
}

int sdx_host_free(void* p) {
  if (p) CK(cudaFreeHost(p), "cudaFreeHost");
  return SDX_OK;
}

int sdx_memcpy_htod_async(sdx_ctx* ctx, sdx_dptr dst, const void* src, size_t bytes, sdx_stream s) {
  USE(ctx);
  CK(cudaMemcpyAsync(reinterpret_cast<void*>(dst), src, bytes, cudaMemcpyHostToDevice, S(ctx, s)), "H2D copy");
  return SDX_OK;
}

int sdx_memcpy_dtoh_async(sdx_ctx* ctx, void* dst, sdx_dptr src, size_t bytes, sdx_stream s) {
  USE(ctx);
  if (inject_fire(FAULT_D2H)) return set_error(SDX_ERR_INJECTED, "injected device-to-host copy fault");
  CK(cudaMemcpyAsync(dst, reinterpret_cast<const void*>(src), bytes, cudaMemcpyDeviceToHost, S(ctx, s)), "D2H copy");
  return SDX_OK;
}

int sdx_memcpy_dtod_async(sdx_ctx* ctx, sdx_dptr dst, sdx_dptr src, size_t bytes, sdx_stream s) {
  USE(ctx);
  CK(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes, cudaMemcpyDeviceToDevice,
                     S(ctx, s)),
     "D2D copy");
  return SDX_OK;
}

int sdx_memset_async(sdx_ctx* ctx, sdx_dptr dst, int value, size_t bytes, sdx_stream s) {
  USE(ctx);
  CK(cudaMemsetAsync(reinterpret_cast<void*>(dst), value, bytes, S(ctx, s)), "memset");
  return SDX_OK;
}

int sdx_stream_create(sdx_ctx* ctx, sdx_stream* out) {
  USE(ctx);
  if (!out) return set_error(SDX_ERR_INVALID, "null out");
  cudaStream_t st;
  CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
  *out = st;
  return SDX_OK;
}

int sdx_stream_destroy(sdx_ctx* ctx, sdx_stream s) {
  if (!ctx) return set_error(SDX_ERR_INVALID, "null context");
  cudaSetDevice(ctx->device);
  if (s) CK(cudaStreamDestroy(static_cast<cudaStream_t>(s)), "cudaStreamDestroy");
  return SDX_OK;
}

static int check_device_word(sdx_ctx* ctx) {
  unsigned int code = 0;
  CK(cudaMemcpy(&code, ctx->err_word, sizeof(code), cudaMemcpyDeviceToHost), "read device error word");
  if (code) {
    ctx->poisoned = 1;
    return set_error(SDX_ERR_DEVICE, "a kernel reported device error 0x%x", code);
  }
  return SDX_OK;
}

int sdx_stream_sync(sdx_ctx* ctx, sdx_stream s, int timeout_ms) {
  USE(ctx);
  if (inject_fire(FAULT_SYNC)) return set_error(SDX_ERR_INJECTED, "injected stream-sync fault");
  cudaStream_t st = S(ctx, s);
  if (timeout_ms > 0) {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      cudaError_t q = cudaStreamQuery(st);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return set_cuda_error(q, "cudaStreamQuery");
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
        return set_error(SDX_ERR_TIMEOUT, "stream still busy after %d ms", timeout_ms);
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  } else {
    CK(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  }
  return check_device_word(ctx);
}

int sdx_stream_query(sdx_ctx* ctx, sdx_stream s, int* done) {
  USE(ctx);
  if (!done) return set_error(SDX_ERR_INVALID, "null out");
  cudaError_t q = cudaStreamQuery(S(ctx, s));
  if (q == cudaSuccess) *done = 1;
  else if (q == cudaErrorNotReady) *done = 0;
  else return set_cuda_error(q, "cudaStreamQuery");
  return SDX_OK;
}

int sdx_event_create(sdx_ctx* ctx, void** ev) {
  USE(ctx);
  cudaEvent_t e;
  CK(cudaEventCreate(&e), "cudaEventCreate");
  *ev = e;
  return SDX_OK;
}

int sdx_event_record(sdx_ctx* ctx, void* ev, sdx_stream s) {
  USE(ctx);
  CK(cudaEventRecord(static_cast<cudaEvent_t>(ev), S(ctx, s)), "cudaEventRecord");
  return SDX_OK;
}

int sdx_event_elapsed_ms(void* start, void* stop, float* ms) {
  CK(cudaEventSynchronize(static_cast<cudaEvent_t>(stop)), "cudaEventSynchronize");
  CK(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop)), "cudaEventElapsedTime");
  return SDX_OK;
}

int sdx_event_destroy(void* ev) {
  if (ev) CK(cudaEventDestroy(static_cast<cudaEvent_t>(ev)), "cudaEventDestroy");
  return SDX_OK;
}

int sdx_graph_begin(sdx_ctx* ctx, sdx_stream s) {
  USE(ctx);
  CK(cudaStreamBeginCapture(S(ctx, s), cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  return SDX_OK;
}

int sdx_graph_end(sdx_ctx* ctx, sdx_stream s, void** graph_exec) {
  USE(ctx);
  cudaGraph_t g;
  CK(cudaStreamEndCapture(S(ctx, s), &g), "cudaStreamEndCapture");
  cudaGraphExec_t ge;
  cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaGraphInstantiate");
  *graph_exec = ge;
  return SDX_OK;
}

int sdx_graph_launch(sdx_ctx* ctx, void* graph_exec, sdx_stream s) {
  USE(ctx);
  if (inject_fire(FAULT_GRAPH)) return set_error(SDX_ERR_INJECTED, "injected graph-launch fault");
  CK(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), S(ctx, s)), "cudaGraphLaunch");
  return SDX_OK;
}

int sdx_graph_destroy(void* graph_exec) {
  if (graph_exec) CK(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)), "cudaGraphExecDestroy");
  return SDX_OK;
}

int sdx_device_error(sdx_ctx* ctx, unsigned int* code) {
  if (!ctx || !code) return set_error(SDX_ERR_INVALID, "null argument");
  cudaSetDevice(ctx->device);
  CK(cudaMemcpy(code, ctx->err_word, sizeof(*code), cudaMemcpyDeviceToHost), "read device error word");
  return SDX_OK;
}

int sdx_clear_device_error(sdx_ctx* ctx) {
  if (!ctx) return set_error(SDX_ERR_INVALID, "null context");
  cudaSetDevice(ctx->device);
  CK(cudaMemset(ctx->err_word, 0, sizeof(unsigned int)), "clear device error word");
  ctx->poisoned = 0;
  return SDX_OK;
}

int sdx_fault_inject(int kind, int nth) {
  std::lock_guard<std::mutex> lk(g_fault_mu);
  g_fault_kind = nth > 0 ? kind : 0;
  g_fault_nth = nth > 0 ? nth : 0;
  g_fault_seen = 0;
  return SDX_OK;
}

uint64_t sdx_launch_count(void) { return g_launches.load(); }

int sdx_selftest_bounded_wait(sdx_ctx* ctx, int wait_ms, sdx_stream s) {
  USE(ctx);
  return bounded_wait_selftest_launch(ctx->err_word, wait_ms, S(ctx, s));
}

// =========================================================================================
// packing + routing
// =========================================================================================
enum Route { R_TC_CONV = 1, R_TC_ROWS = 2, R_DEPTHWISE = 3, R_DIRECT = 4, R_INVALID = 0 };

static int conv_route(const sdx_conv_desc* d) {
  if (d->pad_mode != 0 || d->pad_value != 0.0f) return R_INVALID;
  if (d->group > 1) {
    if (d->group == d->ic && d->oc == d->ic) return R_DEPTHWISE;
    return R_INVALID;
  }
  const bool f16_nhwc = d->x_dtype == SDX_F16 && d->x_layout == SDX_NHWC;
  const bool unit = d->sh == 1 && d->sw == 1;
  if (f16_nhwc && d->ic % 8 == 0 && unit && d->oc >= 8 && d->pool == 0 && d->y_layout == SDX_NHWC &&
      d->add_layout == SDX_NHWC) {
    // 1x1: rows mode (with in_scale: per-image weights, checked at launch)
    if (d->kh == 1 && d->kw == 1 && d->pad_t == 0 && d->pad_l == 0 && d->pad_b == 0 && d->pad_r == 0) return R_TC_ROWS;
    if (d->in_scale == 0) return R_TC_CONV;
  }
  if (d->pool == 0 && d->in_scale == 0) return R_DIRECT;
  // conv + fused 2x2/2 max pool: the small stem convs the reference's GPU plans fuse
  // (GraphCompiler.GpuSmallConv, src/Engine/GraphCompiler.cs:28-32, :897-898): ic < 8, oc a multiple of
  // 8 up to 128, at most 4096 weights, unit strides; NHWC output (the pooled tensor)
  if (d->pool == 1 && d->in_scale == 0 && d->ic < 8 && d->oc % 8 == 0 && d->oc <= 128 &&
      (int64_t)d->oc * d->ic * d->kh * d->kw <= 4096 && unit && d->y_layout == SDX_NHWC && d->add == 0)
    return R_DIRECT;
  return R_INVALID;
}

static int conv_wterms(const sdx_conv_desc* d);

static bool conv_kxn(const sdx_conv_desc* d) {
  // the kx-in-N epilogues read no upsampled residual
  return d->add_up != 2 && tc_conv_kxn(d->kh, d->kw, d->sh, d->sw, d->pad_t, d->pad_l, d->pad_b, d->pad_r, d->oc, d->ic, conv_wterms(d));
}

// Pixel folding factor of a 1x1 tensor-core conv (tc_fold_factor): only for a dense fp16 NHWC
// output and an fp16 residual read at full resolution. Depends on the shape and these layout
// fields only (not on pointers), so sdx_pack_conv and sdx_conv2d agree for one descriptor.
static int conv_fold(const sdx_conv_desc* d) {
  if (conv_route(d) != R_TC_ROWS || d->in_scale) return 1;
  const int64_t ystride = d->y_pix_stride > 0 ? d->y_pix_stride : d->oc;
  if (d->y_dtype != SDX_F16 || ystride != d->oc || d->y_ch_off != 0 || d->add_dtype != SDX_F16 || d->add_up == 2)
    return 1;
  return tc_fold_factor((int64_t)d->batch * d->ih * d->iw, d->ic, d->oc);
}

// fp16 weight terms of a tensor-core conv: the caller's choice, else one for k x k kernels (their thin
// MMAs bound them) and for 1x1 kernels with at least 128 input channels, two (hi + lo) for narrower
// 1x1 kernels. The narrow 1x1 convs sit early in the det/rec trunks, where a weight rounding error
// is shared by every pixel and amplified by every later layer (the squeeze-excitation means shift
// coherently); in the wide ones it averages over the reduction, and their second term doubles the
// MMAs' shared-memory operand traffic, which bounds them.
static int conv_wterms(const sdx_conv_desc* d) {
  if (d->w_terms == 1 || d->w_terms == 2) return d->w_terms;
  if (d->kh * d->kw > 1) return 1;
  return d->ic >= 128 ? 1 : 2;
}

int sdx_pack_conv(const sdx_conv_desc* d, const float* w, void* out, size_t* bytes) {
  if (!d || !bytes) return set_error(SDX_ERR_INVALID, "null argument");
  if (d->w_terms < 0 || d->w_terms > 2) return set_error(SDX_ERR_INVALID, "conv: w_terms must be 0, 1 or 2");
  const int route = conv_route(d);
  const int taps = d->kh * d->kw;
  size_t need = 0;
  switch (route) {
    case R_TC_CONV:
    case R_TC_ROWS:
      need = (route == R_TC_CONV && conv_kxn(d) ? tc_kxn_weights_halves(d->ic, d->oc, conv_wterms(d))
              : conv_fold(d) > 1                ? tc_fold_weights_halves(d->ic, d->oc, conv_fold(d), conv_wterms(d))
                                                : tc_weights_halves(d->oc, d->ic, taps, conv_wterms(d))) *
             sizeof(__half);
      break;
    case R_DEPTHWISE: need = sizeof(float) * (size_t)taps * d->ic; break;
    case R_DIRECT: need = sizeof(float) * (size_t)taps * d->ic * d->oc; break;
    default: return set_error(SDX_ERR_NOT_SUPPORTED, "conv: no CUDA kernel for this shape/flags");
  }
  if (!out) {
    *bytes = need;
    return SDX_OK;
  }
  if (*bytes < need) return set_error(SDX_ERR_INVALID, "pack buffer too small");
  if (!w) return set_error(SDX_ERR_INVALID, "null weights");
  if (route == R_TC_CONV || route == R_TC_ROWS) {
    if (route == R_TC_CONV && conv_kxn(d)) tc_pack_conv_kxn(w, d->oc, d->ic, conv_wterms(d), static_cast<__half*>(out));
    else if (conv_fold(d) > 1) tc_pack_conv_fold(w, d->oc, d->ic, conv_fold(d), conv_wterms(d), static_cast<__half*>(out));
    else tc_pack_conv(w, d->oc, d->ic, d->kh, d->kw, conv_wterms(d), static_cast<__half*>(out));
  } else if (route == R_DEPTHWISE) {
    float* o = static_cast<float*>(out);
    for (int c = 0; c < d->ic; c++)
      for (int t = 0; t < taps; t++) o[(size_t)t * d->ic + c] = w[(size_t)c * taps + t];
  } else {
    float* o = static_cast<float*>(out);  // [tap][ic][oc]
    for (int oc = 0; oc < d->oc; oc++)
      for (int c = 0; c < d->ic; c++)
        for (int t = 0; t < taps; t++) o[((size_t)t * d->ic + c) * d->oc + oc] = w[((size_t)oc * d->ic + c) * taps + t];
  }
  *bytes = need;
  return SDX_OK;
}

int sdx_pack_convt(int ic, int oc, int kh, int kw, const float* w, void* out, size_t* bytes) {
  if (!bytes) return set_error(SDX_ERR_INVALID, "null argument");
  size_t need = oc >= 8 ? tc_convt_weights_halves(ic, oc, kh, kw) * sizeof(__half) : sizeof(float) * (size_t)ic * oc * kh * kw;
  if (!out) {
    *bytes = need;
    return SDX_OK;
  }
  if (*bytes < need) return set_error(SDX_ERR_INVALID, "pack buffer too small");
  if (oc >= 8) tc_pack_convt(w, ic, oc, kh, kw, static_cast<__half*>(out));
  else memcpy(out, w, need);
  *bytes = need;
  return SDX_OK;
}

int sdx_pack_gemm(int k, int n, int trans_b, const float* b, void* out, size_t* bytes) {
  if (!bytes) return set_error(SDX_ERR_INVALID, "null argument");
  size_t need = tc_weights_halves(n, k, 1, 2) * sizeof(__half);
  if (!out) {
    *bytes = need;
    return SDX_OK;
  }
  if (*bytes < need) return set_error(SDX_ERR_INVALID, "pack buffer too small");
  tc_pack_gemm(b, k, n, trans_b, static_cast<__half*>(out));
  *bytes = need;
  return SDX_OK;
}

// Per-image scaled weights of a 1x1 tensor-core conv with in_scale: batch two-term copies of the
// packed weights. The form needs one N tile (oc <= 128) and resident weights (ic <= 256).
size_t sdx_conv_scaled_weights_bytes(const sdx_conv_desc* d) {
  if (!d || conv_route(d) != R_TC_ROWS || d->oc > 128 || d->ic > 256 || d->batch <= 0) return 0;
  int BN, nt;
  tc_plan_n(d->oc, &BN, &nt);
  return (size_t)d->batch * 2 * (size_t)BN * nt * (size_t)tc_kpad_of(d->ic) * sizeof(__half);
}

// =========================================================================================
// ops
// =========================================================================================
int sdx_dw_pw_supported(const sdx_dwpw_desc* d) {
  if (!d) return 0;
  const sdx_conv_desc& w = d->dw;
  const sdx_conv_desc& p = d->pw;
  const bool dw_ok = conv_route(&w) == R_DEPTHWISE && w.kh == 3 && w.kw == 3 && w.sh == 1 && w.sw == 1 &&
                     w.pad_t == 1 && w.pad_l == 1 && w.pad_b == 1 && w.pad_r == 1 && w.x_dtype == SDX_F16 &&
                     w.x_layout == SDX_NHWC && w.y_dtype == SDX_F16 && w.pool == 0 && (w.ic == 64 || w.ic == 128) &&
                     (w.act == SDX_ACT_NONE || w.act == SDX_ACT_RELU || w.act == SDX_ACT_HARDSWISH);
  const int64_t ystride = p.y_pix_stride > 0 ? p.y_pix_stride : p.oc;
  const bool pw_ok = conv_route(&p) == R_TC_ROWS && p.in_scale == 0 && p.ic == w.oc && p.batch == w.batch &&
                     p.ih == w.oh && p.iw == w.ow && p.oc <= 128 && p.y_dtype == SDX_F16 && p.add_up == 0 &&
                     ystride % 8 == 0 && p.y_ch_off % 8 == 0 && (p.oc % 16 == 0);
  return dw_ok && pw_ok ? 1 : 0;
}

int sdx_dw_pw(sdx_ctx* ctx, const sdx_dwpw_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  if (!sdx_dw_pw_supported(d))
    return set_error(SDX_ERR_NOT_SUPPORTED, "dw+pw: needs a 3x3 s1 depthwise over 64 or 128 fp16 channels (act none, relu or "
                                            "hardswish) and a 1x1 conv to at most 128 fp16 outputs (multiples of 16)");
  if (d->pw.add || d->dw.add) return set_error(SDX_ERR_NOT_SUPPORTED, "dw+pw: no residuals");
  if (!d->dw.bias) return set_error(SDX_ERR_INVALID, "dw+pw: depthwise bias required (zeros when absent)");
  const sdx_conv_desc& w = d->dw;
  const sdx_conv_desc& pw = d->pw;
  TcProblem p;
  memset(&p, 0, sizeof(p));
  p.mode = TC_CONV;
  p.a = P<const __half>(w.x);
  p.lda = w.ic;
  p.M = w.batch * w.oh * w.ow;
  p.K = w.ic;
  p.batch = w.batch;
  p.H = w.ih;
  p.W = w.iw;
  p.C = w.ic;
  p.OH = w.oh;
  p.OW = w.ow;
  p.kh = 1;
  p.kw = 1;
  p.w = P<const __half>(pw.w);
  p.wterms = conv_wterms(&pw);
  p.N = pw.oc;
  p.bias = P<const float>(pw.bias);
  p.out = P<void>(pw.y);
  p.out_f32 = 0;
  p.out_pix_stride = pw.y_pix_stride > 0 ? pw.y_pix_stride : pw.oc;
  p.out_ch_off = pw.y_ch_off;
  p.act = pw.act;
  p.gap = P<float>(pw.gap_sums);
  p.err = ctx->err_word;
  p.dw_w = P<const float>(w.w);
  p.dw_b = P<const float>(w.bias);
  p.dw_scale = P<const float>(w.in_scale);
  p.dw_act = w.act;
  return tc_launch(p, S(ctx, s));
}

int sdx_conv2d(sdx_ctx* ctx, const sdx_conv_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  if (d->batch <= 0 || d->oh <= 0 || d->ow <= 0) return set_error(SDX_ERR_INVALID, "conv: empty shape");
  if (d->w_terms < 0 || d->w_terms > 2) return set_error(SDX_ERR_INVALID, "conv: w_terms must be 0, 1 or 2");
  // output size must follow the ONNX formula (src/Engine/GraphCompiler.cs:1790-1794)
  const int oh = (d->ih + d->pad_t + d->pad_b - d->kh) / d->sh + 1, ow = (d->iw + d->pad_l + d->pad_r - d->kw) / d->sw + 1;
  if (oh != d->oh || ow != d->ow) return set_error(SDX_ERR_INVALID, "conv: output %dx%d, expected %dx%d", d->oh, d->ow, oh, ow);
  const int route = conv_route(d);
  if (d->add_up == 2 && route != R_TC_CONV && route != R_TC_ROWS)
    return set_error(SDX_ERR_NOT_SUPPORTED, "conv: upsampled residual only on the tensor-core routes");
  if (d->gap_sums && route != R_TC_ROWS)
    return set_error(SDX_ERR_NOT_SUPPORTED, "conv: fused channel sums only on the 1x1 tensor-core route");
  const int64_t ystride = d->y_pix_stride > 0 ? d->y_pix_stride : d->oc;
  cudaStream_t st = S(ctx, s);
  switch (route) {
    case R_TC_CONV:
    case R_TC_ROWS: {
      TcProblem p;
      memset(&p, 0, sizeof(p));
      p.mode = route == R_TC_CONV ? TC_CONV : TC_ROWS;
      p.a = P<const __half>(d->x);
      p.lda = d->ic;
      p.M = d->batch * d->ih * d->iw;
      p.K = d->ic;
      p.batch = d->batch;
      p.H = d->ih;
      p.W = d->iw;
      p.C = d->ic;
      p.OH = d->oh;
      p.OW = d->ow;
      p.kh = d->kh;
      p.kw = d->kw;
      p.pad_t = d->pad_t;
      p.pad_l = d->pad_l;
      p.w = P<const __half>(d->w);
      p.wterms = conv_wterms(d);
      p.kxn = route == R_TC_CONV && conv_kxn(d) ? 1 : 0;
      p.N = d->oc;
      p.bias = P<const float>(d->bias);
      p.res = P<const void>(d->add);
      p.res_f32 = d->add_dtype == SDX_F32;
      p.res_pix_stride = d->oc;
      if (d->add_up == 2) {
        if (!d->add || d->add_dtype != SDX_F16 || (d->oh & 1) || (d->ow & 1) || d->pool)
          return set_error(SDX_ERR_NOT_SUPPORTED, "conv: upsampled residual needs fp16 add, even oh/ow, no pool");
        p.res_up = 2;
      } else if (d->add_up != 0 && d->add_up != 1) {
        return set_error(SDX_ERR_INVALID, "conv: add_up must be 0, 1 or 2");
      }
      p.res_ch_off = 0;
      p.out = P<void>(d->y);
      p.out_f32 = d->y_dtype == SDX_F32;
      p.out_pix_stride = ystride;
      p.out_ch_off = d->y_ch_off;
      p.act = d->act;
      p.gap = P<float>(d->gap_sums);
      p.err = ctx->err_word;
      if (route == R_TC_ROWS && d->in_scale) {
        // x * s read as x: the weights scaled per image (two terms) into the caller's scratch
        if (!d->w_scaled || sdx_conv_scaled_weights_bytes(d) == 0 || d->gap_sums)
          return set_error(SDX_ERR_NOT_SUPPORTED,
                           "conv: in_scale on a 1x1 conv needs w_scaled scratch, oc <= 128, ic <= 256 and no fused "
                           "channel sums");
        int BN, nt;
        tc_plan_n(d->oc, &BN, &nt);
        const int rc = tc_scale_weights_launch(P<const __half>(d->w), conv_wterms(d), BN * nt, tc_kpad_of(d->ic), d->ic,
                                               P<const float>(d->in_scale), d->batch, P<__half>(d->w_scaled), st);
        if (rc) return rc;
        p.w = P<const __half>(d->w_scaled);
        p.wterms = 2;
        p.img_rows = d->ih * d->iw;
        if (p.img_rows % 128 != 0) p.mode = TC_CONV;  // 128-row tiles would straddle images: pixel tiles
      }
      if (route == R_TC_ROWS) {
        const int f = conv_fold(d);
        if (f > 1) {
          // f consecutive pixels per GEMM row over the same memory (block-diagonal weights)
          p.fold = f;
          p.bias_mod = d->oc;
          p.M /= f;
          p.K *= f;
          p.lda *= f;
          p.N *= f;
          p.res_pix_stride *= f;
          p.out_pix_stride *= f;
        }
      }
      return tc_launch(p, st);
    }
    case R_DEPTHWISE: {
      if (d->x_dtype != SDX_F16 || d->y_dtype != SDX_F16 || d->x_layout != SDX_NHWC || d->pool || ystride != d->oc ||
          (d->add && d->add_dtype != SDX_F16))
        return set_error(SDX_ERR_NOT_SUPPORTED, "depthwise: fp16 NHWC only");
      DwArgs a;
      a.batch = d->batch; a.ih = d->ih; a.iw = d->iw; a.c = d->ic; a.oh = d->oh; a.ow = d->ow;
      a.kh = d->kh; a.kw = d->kw; a.sh = d->sh; a.sw = d->sw; a.pt = d->pad_t; a.pl = d->pad_l; a.act = d->act;
      a.x = P<const __half>(d->x);
      a.w = P<const float>(d->w);
      a.bias = P<const float>(d->bias);
      a.in_scale = P<const float>(d->in_scale);
      a.add = P<const __half>(d->add);
      a.y = P<__half>(d->y);
      a.err = ctx->err_word;
      if (!a.bias) return set_error(SDX_ERR_INVALID, "depthwise: bias required (zeros when absent)");
      return depthwise_launch(a, st);
    }
    case R_DIRECT: {
      DirectArgs a;
      memset(&a, 0, sizeof(a));
      a.pool = d->pool;
      a.pool_relu = d->pool_relu;
      a.batch = d->batch; a.ih = d->ih; a.iw = d->iw; a.ic = d->ic; a.oh = d->oh; a.ow = d->ow; a.oc = d->oc;
      a.kh = d->kh; a.kw = d->kw; a.sh = d->sh; a.sw = d->sw; a.pt = d->pad_t; a.pl = d->pad_l; a.act = d->act;
      a.x = P<const void>(d->x);
      a.x_f32 = d->x_dtype == SDX_F32;
      a.x_nchw = d->x_layout == SDX_NCHW;
      a.w = P<const float>(d->w);
      a.bias = P<const float>(d->bias);
      a.add = P<const void>(d->add);
      a.add_f32 = d->add_dtype == SDX_F32;
      a.add_nchw = d->add_layout == SDX_NCHW;
      a.y = P<void>(d->y);
      a.y_f32 = d->y_dtype == SDX_F32;
      a.y_nchw = d->y_layout == SDX_NCHW;
      a.y_pix_stride = ystride;
      a.y_ch_off = d->y_ch_off;
      a.err = ctx->err_word;
      return direct_conv_launch(a, st);
    }
    default: return set_error(SDX_ERR_NOT_SUPPORTED, "conv: no CUDA kernel for this shape/flags");
  }
}

int sdx_gemm(sdx_ctx* ctx, const sdx_gemm_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  TcProblem p;
  memset(&p, 0, sizeof(p));
  p.mode = TC_ROWS;
  p.a = P<const __half>(d->a);
  p.lda = d->lda > 0 ? d->lda : d->k;
  p.M = d->m;
  p.K = d->k;
  p.w = P<const __half>(d->w);
  p.wterms = 2;
  p.N = d->n;
  p.bias = P<const float>(d->bias);
  p.res = P<const void>(d->add);
  p.res_f32 = d->add_dtype == SDX_F32;
  p.res_pix_stride = d->ldadd > 0 ? d->ldadd : d->n;
  p.out = P<void>(d->y);
  p.out_f32 = d->y_dtype == SDX_F32;
  p.out_pix_stride = d->ldy > 0 ? d->ldy : d->n;
  p.act = d->act;
  p.err = ctx->err_word;
  return tc_launch(p, S(ctx, s));
}

// Scratch of the fused CTC head: per row and 128-column tile the (max, index, denominator) state,
// [n_tiles][m] each, every array 256-byte aligned.
static size_t argmax_part_bytes(int m) { return ((size_t)m * 4 + 255) / 256 * 256; }

size_t sdx_gemm_argmax_scratch_bytes(int m, int n) {
  if (m <= 0 || n <= 0) return 0;
  int BN, nt;
  tc_plan_n(n, &BN, &nt);
  return 3 * (size_t)nt * argmax_part_bytes(m);
}

int sdx_gemm_argmax(sdx_ctx* ctx, const sdx_gemm_argmax_desc* dd, sdx_stream s) {
  USE(ctx);
  if (!dd) return set_error(SDX_ERR_INVALID, "null desc");
  const sdx_gemm_desc* d = &dd->gemm;
  if (d->m <= 0 || d->n <= 0 || d->k <= 0) return set_error(SDX_ERR_INVALID, "gemm argmax: empty problem");
  if (!dd->indices || !dd->probs || !dd->scratch) return set_error(SDX_ERR_INVALID, "gemm argmax: null output or scratch");
  if (d->add || d->act != SDX_ACT_NONE)
    return set_error(SDX_ERR_NOT_SUPPORTED, "gemm argmax: the CTC projection has no residual or activation");
  if (dd->scratch & 255) return set_error(SDX_ERR_INVALID, "gemm argmax: scratch must be 256-byte aligned");
  LAUNCH_GUARD();
  int BN, nt;
  tc_plan_n(d->n, &BN, &nt);
  const size_t part = (size_t)nt * argmax_part_bytes(d->m);
  TcProblem p;
  memset(&p, 0, sizeof(p));
  p.mode = TC_ROWS;
  p.a = P<const __half>(d->a);
  p.lda = d->lda > 0 ? d->lda : d->k;
  p.M = d->m;
  p.K = d->k;
  p.w = P<const __half>(d->w);
  p.wterms = 2;
  p.N = d->n;
  p.bias = P<const float>(d->bias);
  p.act = SDX_ACT_NONE;
  p.out_pix_stride = d->n;
  p.arg_m = P<float>(dd->scratch);
  p.arg_i = P<int>(dd->scratch + part);
  p.arg_s = P<float>(dd->scratch + 2 * part);
  p.arg_ld = (int)(argmax_part_bytes(d->m) / 4);  // tile t's states start at t * arg_ld (256-byte rows)
  p.err = ctx->err_word;
  cudaStream_t st = S(ctx, s);
  int rc = tc_launch(p, st);
  if (rc) return rc;
  return ctc_argmax_merge_launch(p.arg_m, p.arg_i, p.arg_s, d->m, p.arg_ld, nt, P<int>(dd->indices),
                                 P<float>(dd->probs), ctx->err_word, st);
}

int sdx_convt(sdx_ctx* ctx, const sdx_convt_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  if (d->oc >= 8) {
    // a 1x1 implicit GEMM over the input pixels whose epilogue stores each tap's columns as output
    // boxes (see conv_tc.cu)
    if (d->ic % 8 != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "convt: ic must be a multiple of 8");
    TcProblem p;
    memset(&p, 0, sizeof(p));
    p.mode = TC_CONV;
    p.a = P<const __half>(d->x);
    p.lda = d->ic;
    p.M = d->batch * d->ih * d->iw;
    p.K = d->ic;
    p.batch = d->batch;
    p.H = d->ih;
    p.W = d->iw;
    p.C = d->ic;
    p.OH = d->ih;
    p.OW = d->iw;
    p.kh = 1;
    p.kw = 1;
    p.w = P<const __half>(d->w);
    p.wterms = 2;
    p.N = d->kh * d->kw * d->oc;
    p.bias = P<const float>(d->bias);
    p.out = P<void>(d->y);
    p.out_f32 = d->y_dtype == SDX_F32;
    p.out_pix_stride = d->oc;
    p.act = d->act;
    p.convt_kh = d->kh;
    p.convt_kw = d->kw;
    p.convt_oc = d->oc;
    p.convt_H = d->ih;
    p.convt_W = d->iw;
    p.err = ctx->err_word;
    return tc_launch(p, S(ctx, s));
  }
  ConvtDotArgs a;
  a.batch = d->batch; a.ih = d->ih; a.iw = d->iw; a.ic = d->ic; a.oc = d->oc; a.kh = d->kh; a.kw = d->kw;
  a.act = d->act;
  a.y_f32 = d->y_dtype == SDX_F32;
  a.x = P<const __half>(d->x);
  a.w = P<const float>(d->w);
  a.bias = P<const float>(d->bias);
  a.y = P<void>(d->y);
  return convt_dot_launch(a, S(ctx, s));
}

int sdx_convt_chain(sdx_ctx* ctx, const sdx_convt_chain_desc* dd, sdx_stream s) {
  USE(ctx);
  if (!dd) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  const sdx_convt_desc* d = &dd->first;
  if ((d->oc != 8 && d->oc != 16 && d->oc != 24) || d->kh != 2 || d->kw != 2 || dd->oc2 != 1 || dd->kh2 != 2 ||
      dd->kw2 != 2)
    return set_error(SDX_ERR_NOT_SUPPORTED, "convt chain: 2x2 ConvT (8, 16 or 24 outputs) then 2x2 ConvT to one channel");
  if (d->ic % 8 != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "convt chain: ic must be a multiple of 8");
  if (!dd->w2 || !dd->bias2 || !dd->y || !d->x || !d->w) return set_error(SDX_ERR_INVALID, "convt chain: null pointer");
  TcProblem p;
  memset(&p, 0, sizeof(p));
  p.mode = TC_CONV;
  p.a = P<const __half>(d->x);
  p.lda = d->ic;
  p.M = d->batch * d->ih * d->iw;
  p.K = d->ic;
  p.batch = d->batch;
  p.H = d->ih;
  p.W = d->iw;
  p.C = d->ic;
  p.OH = d->ih;
  p.OW = d->iw;
  p.kh = 1;
  p.kw = 1;
  p.w = P<const __half>(d->w);
  p.wterms = 2;
  p.N = d->kh * d->kw * d->oc;
  p.bias = P<const float>(d->bias);
  p.out = nullptr;
  p.out_f32 = 0;
  p.out_pix_stride = d->oc;
  p.act = d->act;
  p.convt_kh = d->kh;
  p.convt_kw = d->kw;
  p.convt_oc = d->oc;
  p.convt_H = d->ih;
  p.convt_W = d->iw;
  p.chain_w2 = P<const float>(dd->w2);
  p.chain_b2 = P<const float>(dd->bias2);
  p.chain_act2 = dd->act2;
  p.chain_y = P<void>(dd->y);
  p.chain_y_f32 = dd->y_dtype == SDX_F32;
  p.err = ctx->err_word;
  return tc_launch(p, S(ctx, s));
}

int sdx_pool(sdx_ctx* ctx, const sdx_pool_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  PoolArgs a;
  a.batch = d->batch; a.ih = d->ih; a.iw = d->iw; a.c = d->c; a.oh = d->oh; a.ow = d->ow; a.kh = d->kh; a.kw = d->kw;
  a.sh = d->sh; a.sw = d->sw; a.pt = d->pad_t; a.pl = d->pad_l; a.is_avg = d->is_avg; a.relu = d->relu;
  a.incl = d->count_include_pad;
  a.x = P<const __half>(d->x);
  a.y = P<__half>(d->y);
  a.x_ps = d->x_pix_stride > 0 ? d->x_pix_stride : d->c;
  a.x_co = d->x_ch_off;
  if (a.x_ps < d->c + d->x_ch_off || a.x_ps % 8 || a.x_co % 8)
    return set_error(SDX_ERR_INVALID, "pool: input slice stride/offset must be multiples of 8 covering c channels");
  return pool_launch(a, S(ctx, s));
}

size_t sdx_channel_gate_scratch_bytes(int batch, int hw, int c) { return gate_scratch_bytes(batch, hw, c); }

int sdx_channel_gate(sdx_ctx* ctx, const sdx_gate_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  GateArgs a;
  a.batch = d->batch; a.hw = d->hw; a.c = d->c; a.r = d->r; a.act1_relu = d->act1_relu; a.hard = d->hard;
  a.alpha = d->alpha; a.beta = d->beta; a.offset = d->offset;
  a.x = P<const __half>(d->x);
  a.w1 = P<const float>(d->w1);
  a.b1 = P<const float>(d->b1);
  a.w2 = P<const float>(d->w2);
  a.b2 = P<const float>(d->b2);
  a.s = P<float>(d->s);
  a.partial = P<float>(d->partial);
  a.sums = P<const float>(d->sums);
  return gate_launch(a, S(ctx, s));
}

int sdx_channel_gate_static(sdx_ctx* ctx, const sdx_gate_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  if (d->batch < 0 || d->hw < 0 || d->c < 0)
    return set_error(SDX_ERR_INVALID, "channel gate (static): negative batch, hw or c");
  const size_t need = gate_scratch_bytes(d->batch, d->hw, d->c);
  if (need > (size_t)SDX_GATE_STATIC_MAX_SCRATCH_BYTES)
    return set_error(SDX_ERR_NOT_SUPPORTED,
                     "channel gate (static): needs %zu scratch bytes, above the fixed %d-byte array; "
                     "use sdx_channel_gate with caller-provided scratch",
                     need, (int)SDX_GATE_STATIC_MAX_SCRATCH_BYTES);
  float* scratch = nullptr;
  int rc = gate_static_scratch(ctx->device, &scratch);
  if (rc) return rc;
  LAUNCH_GUARD();
  GateArgs a;
  a.batch = d->batch; a.hw = d->hw; a.c = d->c; a.r = d->r; a.act1_relu = d->act1_relu; a.hard = d->hard;
  a.alpha = d->alpha; a.beta = d->beta; a.offset = d->offset;
  a.x = P<const __half>(d->x);
  a.w1 = P<const float>(d->w1);
  a.b1 = P<const float>(d->b1);
  a.w2 = P<const float>(d->w2);
  a.b2 = P<const float>(d->b2);
  a.s = P<float>(d->s);
  a.partial = scratch;
  a.sums = P<const float>(d->sums);
  return gate_launch(a, S(ctx, s));
}

int sdx_channel_broadcast(sdx_ctx* ctx, int batch, int64_t pixels, int c, int op, int relu, sdx_dptr x, sdx_dptr v,
                          sdx_dptr y, sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return broadcast_launch(batch, pixels, c, op, relu, P<const __half>(x), P<const float>(v), P<__half>(y), S(ctx, s));
}

int sdx_resize_nearest(sdx_ctx* ctx, const sdx_resize_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  ResizeArgs a;
  a.batch = d->batch; a.ih = d->ih; a.iw = d->iw; a.c = d->c; a.oh = d->oh; a.ow = d->ow; a.add_relu = d->add_relu;
  a.y_pix_stride = d->y_pix_stride > 0 ? d->y_pix_stride : d->c;
  a.y_ch_off = d->y_ch_off;
  a.x = P<const __half>(d->x);
  a.add = P<const __half>(d->add);
  a.y = P<__half>(d->y);
  return resize_launch(a, S(ctx, s));
}

int sdx_concat_channels(sdx_ctx* ctx, int64_t pixels, int nin, const int* counts, const sdx_dptr* ins, sdx_dptr y,
                        sdx_stream s) {
  USE(ctx);
  if (nin <= 0 || nin > 8 || !counts || !ins) return set_error(SDX_ERR_INVALID, "concat: 1..8 inputs");
  LAUNCH_GUARD();
  int total = 0;
  for (int i = 0; i < nin; i++) total += counts[i];
  int off = 0;
  for (int i = 0; i < nin; i++) {
    if (ins[i]) {  // 0: the producer wrote this slice in place
      int rc = slice_copy_launch(pixels, counts[i], P<const __half>(ins[i]), total, off, P<__half>(y), S(ctx, s));
      if (rc) return rc;
    }
    off += counts[i];
  }
  return SDX_OK;
}

int sdx_image_to_tensor(sdx_ctx* ctx, const sdx_image_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  ImageArgs a;
  a.batch = d->batch; a.ih = d->ih; a.iw = d->iw; a.bpp = d->bpp; a.swap = d->swap_rb;
  a.oh = d->oh; a.ow = d->ow; a.pt = d->pad_t; a.pl = d->pad_l; a.y_nhwc_f16 = d->y_nhwc_f16;
  a.stride = d->stride > 0 ? d->stride : (int64_t)d->iw * d->bpp;
  a.img_bytes = d->image_bytes > 0 ? d->image_bytes : a.stride * d->ih;
  a.src = P<const uint8_t>(d->src);
  a.lut = P<const float>(d->lut);
  a.y = P<void>(d->y);
  return image_launch(a, S(ctx, s));
}

int sdx_image_conv(sdx_ctx* ctx, const sdx_image_conv_desc* dd, sdx_stream s) {
  USE(ctx);
  if (!dd) return set_error(SDX_ERR_INVALID, "null desc");
  LAUNCH_GUARD();
  const sdx_image_desc* d = &dd->image;
  const sdx_conv_desc* c = &dd->conv;
  ImageArgs im;
  im.batch = d->batch; im.ih = d->ih; im.iw = d->iw; im.bpp = d->bpp; im.swap = d->swap_rb;
  im.oh = d->oh; im.ow = d->ow; im.pt = d->pad_t; im.pl = d->pad_l; im.y_nhwc_f16 = 0;
  im.stride = d->stride > 0 ? d->stride : (int64_t)d->iw * d->bpp;
  im.img_bytes = d->image_bytes > 0 ? d->image_bytes : im.stride * d->ih;
  im.src = P<const uint8_t>(d->src);
  im.lut = P<const float>(d->lut);
  im.y = nullptr;
  if (im.bpp != 3 && im.bpp != 4) return set_error(SDX_ERR_INVALID, "image conv: 3 or 4 bytes per pixel");
  if (im.ih <= 0 || im.iw <= 0 || im.batch <= 0) return set_error(SDX_ERR_INVALID, "image conv: empty image");
  if (im.stride < (int64_t)im.iw * im.bpp || im.img_bytes < im.stride * im.ih)
    return set_error(SDX_ERR_INVALID, "image conv: stride");
  if (!im.src || !im.lut) return set_error(SDX_ERR_INVALID, "image conv: null pointer");
  if (c->batch != d->batch || c->ih != d->oh || c->iw != d->ow || c->ic != 3 || c->group != 1)
    return set_error(SDX_ERR_INVALID, "image conv: the conv must read the image tensor (batch, 3 x oh x ow)");
  const int oh = (c->ih + c->pad_t + c->pad_b - c->kh) / c->sh + 1, ow = (c->iw + c->pad_l + c->pad_r - c->kw) / c->sw + 1;
  if (oh != c->oh || ow != c->ow) return set_error(SDX_ERR_INVALID, "image conv: output %dx%d, expected %dx%d", c->oh, c->ow, oh, ow);
  DirectArgs a;
  memset(&a, 0, sizeof(a));
  a.batch = c->batch; a.ih = c->ih; a.iw = c->iw; a.ic = c->ic; a.oh = c->oh; a.ow = c->ow; a.oc = c->oc;
  a.kh = c->kh; a.kw = c->kw; a.sh = c->sh; a.sw = c->sw; a.pt = c->pad_t; a.pl = c->pad_l; a.act = c->act;
  a.x = nullptr;
  a.x_f32 = 1;
  a.x_nchw = 1;
  a.w = P<const float>(c->w);
  a.bias = P<const float>(c->bias);
  a.add = P<const void>(c->add);
  a.y = P<void>(c->y);
  a.y_f32 = c->y_dtype == SDX_F32;
  a.y_nchw = c->y_layout == SDX_NCHW;
  a.y_pix_stride = c->y_pix_stride > 0 ? c->y_pix_stride : c->oc;
  a.y_ch_off = c->y_ch_off;
  a.err = ctx->err_word;
  if (!a.w || !a.y) return set_error(SDX_ERR_INVALID, "image conv: null pointer");
  if (c->pool || c->pad_mode != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "image conv: pooled or non-zero-padded conv");
  if (!stem_image_launch(im, a, S(ctx, s)))
    return set_error(SDX_ERR_NOT_SUPPORTED, "image conv: no fused kernel for this conv (run image_to_tensor + conv2d)");
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "stem_image launch");
  count_launch();
  return SDX_OK;
}

int sdx_concat_nearest(sdx_ctx* ctx, int batch, int oh, int ow, int nin, const int* counts, const int* scales,
                       const sdx_dptr* ins, sdx_dptr y, sdx_stream s) {
  USE(ctx);
  if (nin <= 0 || nin > 8 || !counts || !scales || !ins) return set_error(SDX_ERR_INVALID, "concat nearest: 1..8 inputs");
  LAUNCH_GUARD();
  ConcatNearestArgs a;
  memset(&a, 0, sizeof(a));
  a.batch = batch; a.oh = oh; a.ow = ow; a.nin = nin;
  int off = 0;
  for (int i = 0; i < nin; i++) {
    a.c[i] = counts[i];
    a.s[i] = scales[i];
    a.off[i] = off;
    a.x[i] = P<const __half>(ins[i]);
    off += counts[i];
  }
  a.ctot = off;
  a.y = P<__half>(y);
  return concat_nearest_launch(a, S(ctx, s));
}

int sdx_binary(sdx_ctx* ctx, int64_t n, int op, int relu, sdx_dptr a, sdx_dptr b, sdx_dptr y, sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return binary_launch(n, op, relu, P<const __half>(a), P<const __half>(b), P<__half>(y), S(ctx, s));
}

int sdx_act(sdx_ctx* ctx, int64_t n, int act, sdx_dptr x, sdx_dptr y, sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return act_launch(n, act, P<const __half>(x), P<__half>(y), S(ctx, s));
}

int sdx_convert(sdx_ctx* ctx, int batch, int c, int64_t hw, int x_dtype, int x_layout, int y_dtype, int y_layout,
                sdx_dptr x, sdx_dptr y, sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return convert_launch(batch, c, c, hw, x_dtype == SDX_F32, x_layout == SDX_NCHW, y_dtype == SDX_F32,
                        y_layout == SDX_NCHW, P<const void>(x), P<void>(y), S(ctx, s));
}

int sdx_convert_pad(sdx_ctx* ctx, int batch, int c, int c_out, int64_t hw, int x_dtype, int x_layout, int y_dtype,
                    int y_layout, sdx_dptr x, sdx_dptr y, sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return convert_launch(batch, c, c_out, hw, x_dtype == SDX_F32, x_layout == SDX_NCHW, y_dtype == SDX_F32,
                        y_layout == SDX_NCHW, P<const void>(x), P<void>(y), S(ctx, s));
}

int sdx_layernorm(sdx_ctx* ctx, int64_t rows, int c, float eps, sdx_dptr x, sdx_dptr w, sdx_dptr b, sdx_dptr y,
                  sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return layernorm_launch(rows, c, eps, P<const __half>(x), P<const float>(w), P<const float>(b), P<__half>(y), S(ctx, s));
}

int sdx_softmax(sdx_ctx* ctx, int64_t rows, int c, int y_dtype, sdx_dptr x, sdx_dptr y, sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return softmax_launch(rows, c, y_dtype == SDX_F32, P<const __half>(x), P<void>(y), S(ctx, s));
}

int sdx_attention(sdx_ctx* ctx, int batch, int t, int heads, int d, float scale, sdx_dptr qkv, sdx_dptr y,
                  sdx_stream s) {
  USE(ctx);
  LAUNCH_GUARD();
  return attention_launch(batch, t, heads, d, scale, P<const __half>(qkv), P<__half>(y), S(ctx, s));
}

static bool dtype_ok(int t) { return t == SDX_F16 || t == SDX_F32; }

int sdx_binary_bcast(sdx_ctx* ctx, const sdx_bcast_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  if (d->rank < 1 || d->rank > SDX_BCAST_MAX_RANK) return set_error(SDX_ERR_INVALID, "bcast: rank must be 1..6");
  if (d->op < 0 || d->op > 3 || d->act < 0 || d->act > 5) return set_error(SDX_ERR_INVALID, "bcast: bad op or act");
  if (!dtype_ok(d->a_dtype) || !dtype_ok(d->b_dtype) || !dtype_ok(d->y_dtype))
    return set_error(SDX_ERR_INVALID, "bcast: bad dtype");
  if (!d->a || !d->b || !d->y) return set_error(SDX_ERR_INVALID, "bcast: null pointer");
  BcastArgs p;
  memset(&p, 0, sizeof(p));
  p.rank = d->rank;
  int64_t sa = 1, sb = 1, n = 1;
  for (int i = d->rank - 1; i >= 0; i--) {
    const int64_t o = d->out_shape[i], ea = d->a_shape[i], eb = d->b_shape[i];
    if (o < 0 || (ea != o && ea != 1) || (eb != o && eb != 1))
      return set_error(SDX_ERR_INVALID, "bcast: dim %d: %lld vs %lld / %lld do not broadcast", i, (long long)o,
                       (long long)ea, (long long)eb);
    p.shape[i] = o;
    p.sa[i] = ea == 1 ? 0 : sa;
    p.sb[i] = eb == 1 ? 0 : sb;
    sa *= ea;
    sb *= eb;
    n *= o;
  }
  p.n = n;
  p.op = d->op;
  p.act = d->act;
  p.a_f32 = d->a_dtype == SDX_F32;
  p.b_f32 = d->b_dtype == SDX_F32;
  p.y_f32 = d->y_dtype == SDX_F32;
  p.a = P<const void>(d->a);
  p.b = P<const void>(d->b);
  p.y = P<void>(d->y);
  LAUNCH_GUARD();
  return bcast_binary_launch(p, S(ctx, s));
}

int sdx_safe_div(sdx_ctx* ctx, const sdx_safediv_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  if (d->n < 0 || !dtype_ok(d->dtype)) return set_error(SDX_ERR_INVALID, "safediv: bad size or dtype");
  if (!(d->eps > 0.0f)) return set_error(SDX_ERR_INVALID, "safediv: eps must be > 0");
  if (d->n && (!d->a || !d->b || !d->y)) return set_error(SDX_ERR_INVALID, "safediv: null pointer");
  LAUNCH_GUARD();
  return safediv_launch(d->n, d->eps, d->lo, d->hi, d->dtype == SDX_F32, P<const void>(d->a), P<const void>(d->b),
                        P<void>(d->y), S(ctx, s));
}

int sdx_channel_shift(sdx_ctx* ctx, const sdx_shift_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  if (d->batch < 0 || d->h < 0 || d->w < 0 || d->c < 0 || (d->axis != 2 && d->axis != 3) || d->ngroups < 0 ||
      d->ngroups > 8 || !dtype_ok(d->dtype))
    return set_error(SDX_ERR_INVALID, "channel shift: bad shape, axis (2 or 3) or group count (<= 8)");
  ShiftArgs a;
  memset(&a, 0, sizeof(a));
  a.batch = d->batch; a.h = d->h; a.w = d->w; a.c = d->c; a.axis = d->axis; a.ng = d->ngroups;
  int prev = 0;
  for (int g = 0; g < d->ngroups; g++) {
    if (d->group_ends[g] < prev || d->group_ends[g] > d->c)
      return set_error(SDX_ERR_INVALID, "channel shift: group ends must ascend within c");
    a.ends[g] = prev = d->group_ends[g];
    a.offs[g] = d->offsets[g];
  }
  a.f32 = d->dtype == SDX_F32;
  a.x = P<const void>(d->x);
  a.y = P<void>(d->y);
  LAUNCH_GUARD();
  return channel_shift_launch(a, S(ctx, s));
}

int sdx_uphead(sdx_ctx* ctx, const sdx_uphead_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  if (d->batch < 0 || d->ih <= 0 || d->iw <= 0 || d->oh < 0 || d->ow < 0 || !(d->scale_h > 0) || !(d->scale_w > 0) ||
      !dtype_ok(d->x_dtype) || !dtype_ok(d->skip_dtype) || !dtype_ok(d->y_dtype))
    return set_error(SDX_ERR_INVALID, "uphead: bad shape, scale or dtype");
  if (!d->x || !d->skip || !d->w || !d->y) return set_error(SDX_ERR_INVALID, "uphead: null pointer");
  UpHeadArgs a;
  memset(&a, 0, sizeof(a));
  a.batch = d->batch; a.ih = d->ih; a.iw = d->iw; a.c = d->c; a.oh = d->oh; a.ow = d->ow; a.oc = d->oc;
  a.sy = d->scale_h; a.sx = d->scale_w;
  a.resize_relu = d->resize_relu; a.skip_relu = d->skip_relu; a.act = d->act;
  a.x_f32 = d->x_dtype == SDX_F32; a.skip_f32 = d->skip_dtype == SDX_F32; a.y_f32 = d->y_dtype == SDX_F32;
  a.x = P<const void>(d->x);
  a.skip = P<const void>(d->skip);
  a.w = P<const float>(d->w);
  a.bias = P<const float>(d->bias);
  a.y = P<void>(d->y);
  LAUNCH_GUARD();
  return uphead_launch(a, S(ctx, s));
}

int sdx_matmul(sdx_ctx* ctx, const sdx_matmul_desc* d, sdx_stream s) {
  USE(ctx);
  if (!d) return set_error(SDX_ERR_INVALID, "null desc");
  if (d->rank < 2 || d->rank > SDX_BCAST_MAX_RANK || !dtype_ok(d->a_dtype) || !dtype_ok(d->b_dtype) ||
      !dtype_ok(d->y_dtype))
    return set_error(SDX_ERR_INVALID, "matmul: rank must be 2..6; bad dtype");
  const int r = d->rank;
  const int64_t m = d->a_shape[r - 2], k = d->a_shape[r - 1], n = d->b_shape[r - 1];
  if (d->b_shape[r - 2] != k) return set_error(SDX_ERR_INVALID, "matmul: K mismatch");
  if (m > INT32_MAX || k > INT32_MAX || n > INT32_MAX) return set_error(SDX_ERR_NOT_SUPPORTED, "matmul: dims too large");
  MatMulArgs p;
  memset(&p, 0, sizeof(p));
  p.m = (int)m;
  p.k = (int)k;
  p.n = (int)n;
  p.batch_rank = r - 2;
  int64_t batch = 1, as = m * k, bs = k * n;
  for (int i = r - 3; i >= 0; i--) {
    const int64_t ea = d->a_shape[i], eb = d->b_shape[i], o = ea == 1 ? eb : ea;
    if ((ea != o && ea != 1) || (eb != o && eb != 1) || o < 0)
      return set_error(SDX_ERR_INVALID, "matmul: batch dim %d does not broadcast", i);
    p.bshape[i] = o;
    p.a_bstride[i] = ea == 1 ? 0 : as;
    p.b_bstride[i] = eb == 1 ? 0 : bs;
    as *= ea;
    bs *= eb;
    batch *= o;
  }
  if (batch > INT32_MAX) return set_error(SDX_ERR_NOT_SUPPORTED, "matmul: batch too large");
  p.batch = (int)batch;
  p.a_f32 = d->a_dtype == SDX_F32;
  p.b_f32 = d->b_dtype == SDX_F32;
  p.y_f32 = d->y_dtype == SDX_F32;
  p.a = P<const void>(d->a);
  p.b = P<const void>(d->b);
  p.y = P<void>(d->y);
  LAUNCH_GUARD();
  return batched_matmul_launch(p, S(ctx, s));
}

}  // extern "C"
