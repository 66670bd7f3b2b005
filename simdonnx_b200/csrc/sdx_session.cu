// CudaGraphModel + CudaInferenceSession: the node list of one compiled plan over one device arena,
// validated by one eager pass and then captured once into a CUDA graph (the pre-recorded command
// buffer of VkInferenceSession.Record, src/Backends/Vulkan/VkSession.cs:282-337; Run = submit +
// wait, VkSession.cs:535-556). Not thread-safe, like the Vulkan session (VkSession.cs:61).
#include <cuda_runtime.h>

#include <cstring>
#include <new>
#include <vector>

#include "../../include/sdxcuda.h"
#include "sdx_internal.h"

using namespace sdx;

struct sdx_session {
  sdx_ctx* ctx;
  cudaStream_t stream;
  void* arena;
  size_t arena_bytes;
  struct Node {
    int kind;
    std::vector<unsigned char> desc;
  };
  std::vector<Node> nodes;
  sdx_dptr in, out;
  size_t in_bytes, out_bytes;
  cudaGraphExec_t graph;
  int built;
  // pipelined submit/wait: two device staging slots per direction and two copy streams, so the
  // host->device copy of batch i+1 and the device->host copy of batch i-1 overlap the compute of i
  struct Pipe {
    bool ready = false;
    cudaStream_t h2d = nullptr, d2h = nullptr;
    void* stage_in[2] = {nullptr, nullptr};
    void* stage_out[2] = {nullptr, nullptr};
    cudaEvent_t in_landed[2] = {}, in_free[2] = {}, out_ready[2] = {}, out_free[2] = {};
    unsigned long long submitted = 0;
  } pipe;
};

static void pipe_release(sdx_session* s) {
  sdx_session::Pipe& p = s->pipe;
  if (p.h2d) cudaStreamSynchronize(p.h2d);
  if (p.d2h) cudaStreamSynchronize(p.d2h);
  for (int i = 0; i < 2; i++) {
    if (p.stage_in[i]) cudaFree(p.stage_in[i]);
    if (p.stage_out[i]) cudaFree(p.stage_out[i]);
    if (p.in_landed[i]) cudaEventDestroy(p.in_landed[i]);
    if (p.in_free[i]) cudaEventDestroy(p.in_free[i]);
    if (p.out_ready[i]) cudaEventDestroy(p.out_ready[i]);
    if (p.out_free[i]) cudaEventDestroy(p.out_free[i]);
  }
  if (p.h2d) cudaStreamDestroy(p.h2d);
  if (p.d2h) cudaStreamDestroy(p.d2h);
  p = sdx_session::Pipe();
}

static int pipe_setup(sdx_session* s) {
  sdx_session::Pipe& p = s->pipe;
  if (p.ready) return SDX_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking);
  for (int i = 0; i < 2 && e == cudaSuccess; i++) {
    if (s->in_bytes) e = cudaMalloc(&p.stage_in[i], s->in_bytes);
    if (e == cudaSuccess && s->out_bytes) e = cudaMalloc(&p.stage_out[i], s->out_bytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.in_landed[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.in_free[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.out_ready[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.out_free[i], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    pipe_release(s);
    return set_cuda_error(e, "session pipeline setup");
  }
  p.ready = true;
  return SDX_OK;
}

static size_t desc_size(int kind) {
  switch (kind) {
    case SDX_OP_CONV: return sizeof(sdx_conv_desc);
    case SDX_OP_GEMM: return sizeof(sdx_gemm_desc);
    case SDX_OP_CONVT: return sizeof(sdx_convt_desc);
    case SDX_OP_POOL: return sizeof(sdx_pool_desc);
    case SDX_OP_CHANNEL_GATE: return sizeof(sdx_gate_desc);
    case SDX_OP_RESIZE_NEAREST: return sizeof(sdx_resize_desc);
    case SDX_OP_CHANNEL_BROADCAST:
    case SDX_OP_CONCAT:
    case SDX_OP_BINARY:
    case SDX_OP_ACT:
    case SDX_OP_CONVERT:
    case SDX_OP_LAYERNORM:
    case SDX_OP_SOFTMAX:
    case SDX_OP_ATTENTION:
    case SDX_OP_CONCAT_NEAREST: return sizeof(sdx_misc_desc);
    case SDX_OP_IMAGE: return sizeof(sdx_image_desc);
    case SDX_OP_IMAGE_CONV: return sizeof(sdx_image_conv_desc);
    case SDX_OP_CONVT_CHAIN: return sizeof(sdx_convt_chain_desc);
    case SDX_OP_BINARY_BCAST: return sizeof(sdx_bcast_desc);
    case SDX_OP_SAFE_DIV: return sizeof(sdx_safediv_desc);
    case SDX_OP_CHANNEL_SHIFT: return sizeof(sdx_shift_desc);
    case SDX_OP_UPHEAD: return sizeof(sdx_uphead_desc);
    case SDX_OP_MATMUL: return sizeof(sdx_matmul_desc);
    case SDX_OP_GEMM_ARGMAX: return sizeof(sdx_gemm_argmax_desc);
    case SDX_OP_DW_PW: return sizeof(sdx_dwpw_desc);
    default: return 0;
  }
}

static int run_node(sdx_session* s, const sdx_session::Node& n) {
  sdx_ctx* c = s->ctx;
  sdx_stream st = s->stream;
  const void* d = n.desc.data();
  const sdx_misc_desc* m = static_cast<const sdx_misc_desc*>(d);
  switch (n.kind) {
    case SDX_OP_CONV: return sdx_conv2d(c, static_cast<const sdx_conv_desc*>(d), st);
    case SDX_OP_GEMM: return sdx_gemm(c, static_cast<const sdx_gemm_desc*>(d), st);
    case SDX_OP_CONVT: return sdx_convt(c, static_cast<const sdx_convt_desc*>(d), st);
    case SDX_OP_POOL: return sdx_pool(c, static_cast<const sdx_pool_desc*>(d), st);
    case SDX_OP_CHANNEL_GATE: return sdx_channel_gate(c, static_cast<const sdx_gate_desc*>(d), st);
    case SDX_OP_RESIZE_NEAREST: return sdx_resize_nearest(c, static_cast<const sdx_resize_desc*>(d), st);
    case SDX_OP_CHANNEL_BROADCAST: return sdx_channel_broadcast(c, m->batch, m->pixels, m->c, m->op, m->relu, m->x, m->b, m->y, st);
    case SDX_OP_CONCAT: return sdx_concat_channels(c, m->pixels, m->nin, m->counts, m->ins, m->y, st);
    case SDX_OP_IMAGE: return sdx_image_to_tensor(c, static_cast<const sdx_image_desc*>(d), st);
    case SDX_OP_IMAGE_CONV: return sdx_image_conv(c, static_cast<const sdx_image_conv_desc*>(d), st);
    case SDX_OP_CONVT_CHAIN: return sdx_convt_chain(c, static_cast<const sdx_convt_chain_desc*>(d), st);
    case SDX_OP_CONCAT_NEAREST:
      return sdx_concat_nearest(c, m->batch, (int)m->rows, (int)m->n, m->nin, m->counts, m->aux, m->ins, m->y, st);
    case SDX_OP_BINARY: return sdx_binary(c, m->n, m->op, m->relu, m->a, m->b, m->y, st);
    case SDX_OP_ACT: return sdx_act(c, m->n, m->act, m->x, m->y, st);
    case SDX_OP_CONVERT:
      return sdx_convert_pad(c, m->batch, m->c, m->aux[0] > 0 ? m->aux[0] : m->c, m->pixels, m->x_dtype, m->x_layout,
                             m->y_dtype, m->y_layout, m->x, m->y, st);
    case SDX_OP_LAYERNORM: return sdx_layernorm(c, m->rows, m->c, m->eps, m->x, m->w, m->bias, m->y, st);
    case SDX_OP_SOFTMAX: return sdx_softmax(c, m->rows, m->c, m->y_dtype, m->x, m->y, st);
    case SDX_OP_ATTENTION: return sdx_attention(c, m->batch, m->t, m->heads, m->d, m->scale, m->x, m->y, st);
    case SDX_OP_BINARY_BCAST: return sdx_binary_bcast(c, static_cast<const sdx_bcast_desc*>(d), st);
    case SDX_OP_SAFE_DIV: return sdx_safe_div(c, static_cast<const sdx_safediv_desc*>(d), st);
    case SDX_OP_CHANNEL_SHIFT: return sdx_channel_shift(c, static_cast<const sdx_shift_desc*>(d), st);
    case SDX_OP_UPHEAD: return sdx_uphead(c, static_cast<const sdx_uphead_desc*>(d), st);
    case SDX_OP_MATMUL: return sdx_matmul(c, static_cast<const sdx_matmul_desc*>(d), st);
    case SDX_OP_GEMM_ARGMAX: return sdx_gemm_argmax(c, static_cast<const sdx_gemm_argmax_desc*>(d), st);
    case SDX_OP_DW_PW: return sdx_dw_pw(c, static_cast<const sdx_dwpw_desc*>(d), st);
    default: return set_error(SDX_ERR_INVALID, "unknown op kind %d", n.kind);
  }
}

static int run_all(sdx_session* s) {
  for (size_t i = 0; i < s->nodes.size(); i++) {
    int rc = run_node(s, s->nodes[i]);
    if (rc) return rc;
  }
  return SDX_OK;
}

extern "C" {

size_t sdx_desc_size(int op_kind) { return desc_size(op_kind); }

int sdx_session_create(sdx_ctx* ctx, size_t arena_bytes, sdx_session** out) {
  if (!ctx || !out) return set_error(SDX_ERR_INVALID, "null argument");
  if (ctx->poisoned) return set_error(SDX_ERR_POISONED, "context saw a device error; close and reopen it");
  cudaSetDevice(ctx->device);
  sdx_session* s = new (std::nothrow) sdx_session();
  if (!s) return set_error(SDX_ERR_OOM, "session allocation");
  s->ctx = ctx;
  s->arena = nullptr;
  s->arena_bytes = arena_bytes;
  s->graph = nullptr;
  s->built = 0;
  s->in = s->out = 0;
  s->in_bytes = s->out_bytes = 0;
  if (inject_fire(FAULT_MALLOC)) {
    delete s;
    return set_error(SDX_ERR_INJECTED, "injected allocation fault");
  }
  cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete s;
    return set_cuda_error(e, "session stream");
  }
  if (arena_bytes) {
    e = cudaMalloc(&s->arena, arena_bytes);
    if (e != cudaSuccess) {
      cudaStreamDestroy(s->stream);
      delete s;
      return set_cuda_error(e, "session arena");
    }
  }
  *out = s;
  return SDX_OK;
}

int sdx_session_arena(sdx_session* s, sdx_dptr* base, size_t* bytes) {
  if (!s) return set_error(SDX_ERR_INVALID, "null session");
  if (base) *base = reinterpret_cast<sdx_dptr>(s->arena);
  if (bytes) *bytes = s->arena_bytes;
  return SDX_OK;
}

int sdx_session_add_node(sdx_session* s, int op_kind, const void* desc, size_t desc_bytes) {
  if (!s || !desc) return set_error(SDX_ERR_INVALID, "null argument");
  if (s->built) return set_error(SDX_ERR_INVALID, "session already built");
  size_t want = desc_size(op_kind);
  if (!want || desc_bytes != want) return set_error(SDX_ERR_INVALID, "op %d: descriptor is %zu bytes, expected %zu", op_kind, desc_bytes, want);
  sdx_session::Node n;
  n.kind = op_kind;
  n.desc.assign(static_cast<const unsigned char*>(desc), static_cast<const unsigned char*>(desc) + desc_bytes);
  s->nodes.push_back(std::move(n));
  return SDX_OK;
}

int sdx_session_set_io(sdx_session* s, sdx_dptr in, size_t in_bytes, sdx_dptr out, size_t out_bytes) {
  if (!s) return set_error(SDX_ERR_INVALID, "null session");
  s->in = in;
  s->in_bytes = in_bytes;
  s->out = out;
  s->out_bytes = out_bytes;
  return SDX_OK;
}

int sdx_session_build(sdx_session* s, int use_graph) {
  if (!s) return set_error(SDX_ERR_INVALID, "null session");
  cudaSetDevice(s->ctx->device);
  // one eager pass validates every node (and sets kernel attributes outside any capture)
  int rc = run_all(s);
  if (rc) return rc;
  rc = sdx_stream_sync(s->ctx, s->stream, 0);
  if (rc) return rc;
  if (use_graph) {
    cudaError_t e = cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaStreamBeginCapture");
    rc = run_all(s);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(s->stream, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return set_cuda_error(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&s->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaGraphInstantiate");
  }
  s->built = 1;
  return SDX_OK;
}

int sdx_session_stream(sdx_session* s, sdx_stream* stream) {
  if (!s || !stream) return set_error(SDX_ERR_INVALID, "null argument");
  *stream = s->stream;
  return SDX_OK;
}

int sdx_session_enqueue(sdx_session* s) {
  if (!s || !s->built) return set_error(SDX_ERR_INVALID, "session not built");
  if (s->ctx->poisoned) return set_error(SDX_ERR_POISONED, "context saw a device error; close and reopen it");
  cudaSetDevice(s->ctx->device);
  if (s->graph) {
    if (inject_fire(FAULT_GRAPH)) return set_error(SDX_ERR_INJECTED, "injected graph-launch fault");
    cudaError_t e = cudaGraphLaunch(s->graph, s->stream);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaGraphLaunch");
    return SDX_OK;
  }
  return run_all(s);
}

int sdx_session_run(sdx_session* s, const void* host_in, void* host_out, int timeout_ms) {
  if (!s || !s->built) return set_error(SDX_ERR_INVALID, "session not built");
  int rc;
  if (host_in && s->in_bytes) {
    rc = sdx_memcpy_htod_async(s->ctx, s->in, host_in, s->in_bytes, s->stream);
    if (rc) return rc;
  }
  rc = sdx_session_enqueue(s);
  if (rc) return rc;
  if (host_out && s->out_bytes) {
    rc = sdx_memcpy_dtoh_async(s->ctx, host_out, s->out, s->out_bytes, s->stream);
    if (rc) return rc;
  }
  return sdx_stream_sync(s->ctx, s->stream, timeout_ms);
}

int sdx_session_node_count(sdx_session* s, int* count) {
  if (!s || !count) return set_error(SDX_ERR_INVALID, "null argument");
  *count = (int)s->nodes.size();
  return SDX_OK;
}

int sdx_session_enqueue_node(sdx_session* s, int index) {
  if (!s) return set_error(SDX_ERR_INVALID, "null session");
  if (index < 0 || index >= (int)s->nodes.size()) return set_error(SDX_ERR_INVALID, "node index %d out of range", index);
  cudaSetDevice(s->ctx->device);
  return run_node(s, s->nodes[(size_t)index]);
}

int sdx_session_submit(sdx_session* s, const void* host_in, void* host_out) {
  if (!s || !s->built) return set_error(SDX_ERR_INVALID, "session not built");
  if (s->ctx->poisoned) return set_error(SDX_ERR_POISONED, "context saw a device error; close and reopen it");
  cudaSetDevice(s->ctx->device);
  int rc = pipe_setup(s);
  if (rc) return rc;
  sdx_session::Pipe& p = s->pipe;
  const int slot = (int)(p.submitted & 1u);
  const bool reuse = p.submitted >= 2;  // the slot's events were recorded by submission i-2
#define PCK(call, what)                                         \
  do {                                                          \
    cudaError_t e_ = (call);                                    \
    if (e_ != cudaSuccess) return set_cuda_error(e_, what);     \
  } while (0)
  if (host_in && s->in_bytes) {
    // the staging slot is free once submission i-2 copied it into the arena
    if (reuse) PCK(cudaStreamWaitEvent(p.h2d, p.in_free[slot], 0), "wait input slot");
    rc = sdx_memcpy_htod_async(s->ctx, reinterpret_cast<sdx_dptr>(p.stage_in[slot]), host_in, s->in_bytes, p.h2d);
    if (rc) return rc;
    PCK(cudaEventRecord(p.in_landed[slot], p.h2d), "record input landed");
    PCK(cudaStreamWaitEvent(s->stream, p.in_landed[slot], 0), "wait input landed");
    PCK(cudaMemcpyAsync(reinterpret_cast<void*>(s->in), p.stage_in[slot], s->in_bytes, cudaMemcpyDeviceToDevice,
                        s->stream), "input into the arena");
    PCK(cudaEventRecord(p.in_free[slot], s->stream), "record input slot free");
  }
  rc = sdx_session_enqueue(s);
  if (rc) return rc;
  if (host_out && s->out_bytes) {
    if (reuse) PCK(cudaStreamWaitEvent(s->stream, p.out_free[slot], 0), "wait output slot");
    PCK(cudaMemcpyAsync(p.stage_out[slot], reinterpret_cast<void*>(s->out), s->out_bytes, cudaMemcpyDeviceToDevice,
                        s->stream), "output out of the arena");
    PCK(cudaEventRecord(p.out_ready[slot], s->stream), "record output ready");
    PCK(cudaStreamWaitEvent(p.d2h, p.out_ready[slot], 0), "wait output ready");
    rc = sdx_memcpy_dtoh_async(s->ctx, host_out, reinterpret_cast<sdx_dptr>(p.stage_out[slot]), s->out_bytes, p.d2h);
    if (rc) return rc;
    PCK(cudaEventRecord(p.out_free[slot], p.d2h), "record output slot free");
  }
#undef PCK
  p.submitted++;
  return SDX_OK;
}

int sdx_session_wait(sdx_session* s, int timeout_ms) {
  if (!s) return set_error(SDX_ERR_INVALID, "null session");
  cudaSetDevice(s->ctx->device);
  int rc = sdx_stream_sync(s->ctx, s->stream, timeout_ms);
  if (rc) return rc;
  if (s->pipe.ready) {
    rc = sdx_stream_sync(s->ctx, s->pipe.d2h, timeout_ms);
    if (rc) return rc;
    rc = sdx_stream_sync(s->ctx, s->pipe.h2d, timeout_ms);
  }
  return rc;
}

int sdx_session_destroy(sdx_session* s) {
  if (!s) return SDX_OK;
  cudaSetDevice(s->ctx->device);
  pipe_release(s);
  cudaStreamSynchronize(s->stream);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  if (s->arena) cudaFree(s->arena);
  cudaStreamDestroy(s->stream);
  delete s;
  return SDX_OK;
}

}  // extern "C"
