// Whole-model executor: loads an engine file (a plan of fused nodes plus a
// packed weight blob), keeps every activation in one device arena and runs
// the node loop, eagerly or as a replayed CUDA graph.  Included by
// snn_api.cu (same translation unit: shares fail() and ensure_init()).
//
// Counterparts in the reference: the node loop and CUDA graph of
// sengine/csrc/cpp_executor.cu (sengine_execute :883-1194,
// sengine_capture_graph / sengine_replay :1270-1293) and the engine-file
// loader of sengine/csrc/sengine_exec.cu (load_plan :516).  The reference's
// file (sengine/build/sengine_io.py:33-38: "SENG", JSON header + weight
// blobs) binds TileLang kernels rebuilt from tuning caches; this file binds
// the fixed fused kernels of this library, so it has its own layout:
//
//   header   SnnEngineHeader (64 bytes)
//   tensors  n_tensors x SnnEngineTensor (16 bytes): byte size and dtype
//   nodes    n_nodes x SnnEngineNode (160 bytes), in execution order
//   blob     blob_bytes: packed 2:4 weights, BN scale/bias, stem and FC
//            parameters, each at a 256-byte aligned offset
//
// All integers little-endian.  Node kinds and their fields:
//   STEM        in0 = images (fp32 NCHW, Tin x B), out; desc; p0 = w, p1 = scale,
//               p2 = bias (fp32); i[0] = Tin; in1 = none, or the spike output of
//               the dual form (out = fp16 BN output, in1 = spikes of
//               desc.neuron on it)
//   CONV        in0 = data, in1 = residual or none, out; desc (no membrane
//               flags: the membrane starts at zero every forward); p0 = packed
//               weights, p1 = scale, p2 = bias
//   HEAD        in0 = features, out = logits; p0 = fc_w, p1 = fc_b;
//               i[0..4] = T, B, HW, C, NC
//   ADD_LIF     in0, in1, out; desc
//   MAXPOOL_LIF in0, out; desc (KH = window, stride, pad; neuron NONE: the
//               plain max pool)
//   LIF         in0, out; desc (the neuron of one input)
//   CONV_TSPLIT as CONV, in the timestep-split form; i[0] = the fp32
//               workspace tensor
//   ATTN        in0 = q, in1 = k, i[0] = v, out; desc T, B, tau,
//               v_threshold, v_reset, tau2 = the attention scale;
//               i[1..3] = tokens, heads, head_dim; desc flags
//               SNN_FLAG_QKV_PACKED: in0 = in1 = i[0] = one q|k|v tensor
// Stem nodes may have no neuron (fp16 BN output); conv nodes may carry the
// dense-weight and general-kernel flags and the fp16 BN output, but never
// the membrane flags (every forward starts from zero).
#pragma once
#include <cstdio>
#include <vector>

namespace {

constexpr char kEngineMagic[4] = {'S', 'N', 'N', 'E'};
constexpr uint32_t kEngineVersion = 2;
constexpr uint32_t kNoTensor = 0xffffffffu;
enum EngineOp : uint32_t { kOpStem = 1, kOpConv = 2, kOpHead = 3, kOpAddLif = 4, kOpMaxPoolLif = 5,
                           kOpLif = 6, kOpAttn = 7, kOpConvTsplit = 8 };

struct SnnEngineHeader {
  char magic[4];
  uint32_t version;
  uint32_t n_tensors, n_nodes;
  uint32_t input, output;      // tensor ids of the images and the logits
  uint32_t T, B;
  uint64_t blob_bytes;
  uint64_t file_bytes;
  uint32_t reserved[4];
};
struct SnnEngineTensor {
  uint64_t bytes;
  uint32_t dtype;              // 0 fp16, 1 fp32
  uint32_t pad;
};
struct SnnEngineNode {
  uint32_t op;
  uint32_t in0, in1, out;
  snn_conv_desc desc;
  uint64_t p0, p1, p2, p3;     // blob offsets
  int32_t i[5];
  uint32_t pad[3];
};
static_assert(sizeof(SnnEngineHeader) == 64, "engine header layout");
static_assert(sizeof(SnnEngineTensor) == 16, "engine tensor record layout");
static_assert(sizeof(SnnEngineNode) == 160, "engine node record layout");

// Reads and validates an engine file on the host (no device use).
int parse_engine_file(const char* path, SnnEngineHeader* h, std::vector<SnnEngineTensor>* tensors,
                      std::vector<SnnEngineNode>* nodes, std::vector<uint8_t>* blob) {
  if (!path) return fail(SNN_E_INVALID, "engine path is null");
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(SNN_E_INVALID, "cannot open engine file %s", path);
  struct Closer { FILE* f; ~Closer() { std::fclose(f); } } closer{f};
  std::fseek(f, 0, SEEK_END);
  const long size = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  if (size < static_cast<long>(sizeof(SnnEngineHeader)) || std::fread(h, sizeof(*h), 1, f) != 1)
    return fail(SNN_E_INVALID, "engine file too short");
  if (std::memcmp(h->magic, kEngineMagic, 4) != 0) return fail(SNN_E_INVALID, "not an engine file (magic)");
  if (h->version != kEngineVersion)
    return fail(SNN_E_INVALID, "engine file version %u (this library reads %u)", h->version, kEngineVersion);
  if (h->n_tensors == 0 || h->n_tensors > 4096 || h->n_nodes == 0 || h->n_nodes > 4096)
    return fail(SNN_E_INVALID, "engine file: bad tensor or node count");
  const uint64_t expect = sizeof(SnnEngineHeader) + uint64_t(h->n_tensors) * sizeof(SnnEngineTensor) +
                          uint64_t(h->n_nodes) * sizeof(SnnEngineNode) + h->blob_bytes;
  if (h->file_bytes != expect || static_cast<uint64_t>(size) != expect)
    return fail(SNN_E_INVALID, "engine file size %ld does not match its header (%llu)", size,
                static_cast<unsigned long long>(expect));
  tensors->resize(h->n_tensors);
  nodes->resize(h->n_nodes);
  blob->resize(h->blob_bytes);
  if (std::fread(tensors->data(), sizeof(SnnEngineTensor), h->n_tensors, f) != h->n_tensors ||
      std::fread(nodes->data(), sizeof(SnnEngineNode), h->n_nodes, f) != h->n_nodes ||
      (h->blob_bytes && std::fread(blob->data(), 1, h->blob_bytes, f) != h->blob_bytes))
    return fail(SNN_E_INVALID, "engine file: short read");
  auto tid_ok = [&](uint32_t t) { return t < h->n_tensors; };
  if (!tid_ok(h->input) || !tid_ok(h->output)) return fail(SNN_E_INVALID, "engine file: bad input/output id");
  if ((*tensors)[h->input].dtype != 1 || (*tensors)[h->output].dtype != 1)
    return fail(SNN_E_INVALID, "engine file: images and logits must be fp32");
  auto off_ok = [&](uint64_t off, uint64_t bytes) {
    return off % 16 == 0 && off <= h->blob_bytes && bytes <= h->blob_bytes - off;
  };
  for (uint32_t n = 0; n < h->n_nodes; ++n) {
    const SnnEngineNode& nd = (*nodes)[n];
    const snn_conv_desc& d = nd.desc;
    if (!tid_ok(nd.in0) || !tid_ok(nd.out) || (nd.in1 != kNoTensor && !tid_ok(nd.in1)))
      return fail(SNN_E_INVALID, "engine node %u: bad tensor id", n);
    const uint64_t in_bytes = (*tensors)[nd.in0].bytes, out_bytes = (*tensors)[nd.out].bytes;
    switch (nd.op) {
      case kOpStem: {
        // Output extent exactly as snn_stem_forward computes it (any pad >= 0
        // and stride >= 1), from dimensions checked positive first.
        if (d.T < 1 || d.B < 1 || d.H < 1 || d.W < 1 || d.Cin < 1 || d.Cout < 1 || d.KH < 1 ||
            d.KW < 1 || d.stride < 1 || d.pad < 0)
          return fail(SNN_E_INVALID, "engine node %u (stem): non-positive dimension", n);
        const int64_t oh = (int64_t(d.H) + 2 * d.pad - d.KH) / d.stride + 1;
        const int64_t ow = (int64_t(d.W) + 2 * d.pad - d.KW) / d.stride + 1;
        if (oh < 1 || ow < 1) return fail(SNN_E_INVALID, "engine node %u (stem): empty output", n);
        const uint64_t px = uint64_t(d.B) * d.H * d.W;
        // SNN_FLAG_SPIKE_BITS: the spikes leave bit-packed, Cout/8 bytes a pixel.
        const uint64_t px_bytes = (d.flags & SNN_FLAG_SPIKE_BITS) ? uint64_t(d.Cout) / 8 : uint64_t(d.Cout) * 2;
        if (nd.i[0] < 1 || in_bytes < uint64_t(nd.i[0]) * d.Cin * px * 4 ||
            out_bytes < uint64_t(d.T) * d.B * uint64_t(oh) * uint64_t(ow) * px_bytes ||
            !off_ok(nd.p0, uint64_t(d.Cout) * d.Cin * d.KH * d.KW * 4) ||
            !off_ok(nd.p1, uint64_t(d.Cout) * 4) || !off_ok(nd.p2, uint64_t(d.Cout) * 4))
          return fail(SNN_E_INVALID, "engine node %u (stem): sizes or offsets out of range", n);
        if (nd.in1 != kNoTensor &&
            (nd.in1 == nd.out || nd.in1 == nd.in0 ||
             (*tensors)[nd.in1].bytes < uint64_t(d.T) * d.B * uint64_t(oh) * uint64_t(ow) * d.Cout * 2))
          return fail(SNN_E_INVALID, "engine node %u (stem): bad spike output tensor", n);
        break;
      }
      case kOpConv:
      case kOpConvTsplit: {
        int32_t oh = 0, ow = 0;
        size_t wbytes = 0;
        int st = snn_conv_out_shape(&d, &oh, &ow);
        if (!st) st = snn_conv_weight_bytes(&d, &wbytes);
        if (st) return st;
        if (nd.op == kOpConvTsplit) {
          size_t ws = 0;
          const uint32_t ws_id = static_cast<uint32_t>(nd.i[0]);
          if ((st = snn_conv_tsplit_workspace_bytes(&d, &ws))) return st;
          if (!tid_ok(ws_id) || (*tensors)[ws_id].bytes < ws)
            return fail(SNN_E_INVALID, "engine node %u (conv): workspace missing or too small", n);
        }
        const uint64_t out_need = uint64_t(d.T) * d.B * oh * ow * d.Cout * (d.neuron == SNN_NEURON_NONE ? 4 : 2);
        if (in_bytes < uint64_t(d.T) * d.B * d.H * d.W * d.Cin * 2 || out_bytes < out_need ||
            (nd.in1 != kNoTensor && (*tensors)[nd.in1].bytes < uint64_t(d.T) * d.B * oh * ow * d.Cout * 2) ||
            !off_ok(nd.p0, wbytes) || !off_ok(nd.p1, uint64_t(d.Cout) * 4) ||
            !off_ok(nd.p2, uint64_t(d.Cout) * 4) ||
            (d.flags & ~(SNN_FLAG_FORCE_GENERIC | SNN_FLAG_DENSE)) != 0 ||
            d.res_mode == SNN_RES_TWO_NEURON || (d.res_mode == SNN_RES_ADD_BEFORE && nd.in1 == kNoTensor))
          return fail(SNN_E_INVALID, "engine node %u (conv): sizes, offsets or flags out of range", n);
        break;
      }
      case kOpHead: {
        const int32_t* i = nd.i;
        if (i[0] < 1 || i[1] < 1 || i[2] < 1 || i[3] < 1 || i[4] < 1 ||
            in_bytes < uint64_t(i[0]) * i[1] * i[2] * i[3] * 2 || out_bytes < uint64_t(i[1]) * i[4] * 4 ||
            !off_ok(nd.p0, uint64_t(i[4]) * i[3] * 4) || !off_ok(nd.p1, uint64_t(i[4]) * 4))
          return fail(SNN_E_INVALID, "engine node %u (head): sizes or offsets out of range", n);
        break;
      }
      case kOpAttn: {
        const int32_t N = nd.i[1], heads = nd.i[2], hd = nd.i[3];
        const uint32_t v_id = static_cast<uint32_t>(nd.i[0]);
        // SNN_FLAG_QKV_PACKED: in0 is one [T*B][N][3C] tensor (in1 and the
        // v id name the same tensor).
        const bool packed = d.flags == SNN_FLAG_QKV_PACKED;
        if (d.T < 1 || d.B < 1 || N < 1 || heads < 1 || (hd != 32 && hd != 64) ||
            (d.flags != 0 && !packed) || nd.in1 == kNoTensor || !tid_ok(v_id) ||
            (packed && (nd.in1 != nd.in0 || v_id != nd.in0)))
          return fail(SNN_E_INVALID, "engine node %u (attention): bad shape, flags or tensor", n);
        const uint64_t need = uint64_t(d.T) * d.B * N * heads * hd * 2;
        const uint64_t in_need = packed ? 3 * need : need;
        if (in_bytes < in_need || out_bytes < need || (*tensors)[nd.in1].bytes < in_need ||
            (*tensors)[v_id].bytes < in_need)
          return fail(SNN_E_INVALID, "engine node %u (attention): sizes out of range", n);
        break;
      }
      case kOpLif:
      case kOpAddLif:
      case kOpMaxPoolLif: {
        // The max pool may read bit-packed spikes (SNN_FLAG_SPIKE_BITS, Cout/8 bytes a pixel).
        const bool bits = nd.op == kOpMaxPoolLif && d.flags == SNN_FLAG_SPIKE_BITS;
        if (d.T < 1 || d.B < 1 || d.H < 1 || d.W < 1 || d.Cout < 1 || (d.flags != 0 && !bits))
          return fail(SNN_E_INVALID, "engine node %u (glue): bad shape or flags", n);
        const uint64_t in_need = uint64_t(d.T) * d.B * d.H * d.W * (bits ? uint64_t(d.Cout) / 8 : uint64_t(d.Cout) * 2);
        uint64_t out_need = uint64_t(d.T) * d.B * d.H * d.W * d.Cout * 2;
        if (nd.op == kOpMaxPoolLif) {
          if (d.KH < 1 || d.KW < 1 || d.stride < 1 || d.pad < 0)
            return fail(SNN_E_INVALID, "engine node %u (maxpool): bad window", n);
          const int64_t oh = (int64_t(d.H) + 2 * d.pad - d.KH) / d.stride + 1;
          const int64_t ow = (int64_t(d.W) + 2 * d.pad - d.KW) / d.stride + 1;
          if (oh < 1 || ow < 1) return fail(SNN_E_INVALID, "engine node %u (maxpool): empty output", n);
          out_need = uint64_t(d.T) * d.B * oh * ow * d.Cout * 2;
        }
        if (in_bytes < in_need || out_bytes < out_need ||
            (nd.op == kOpAddLif && (nd.in1 == kNoTensor || (*tensors)[nd.in1].bytes < in_need)))
          return fail(SNN_E_INVALID, "engine node %u (glue): sizes out of range", n);
        break;
      }
      default:
        return fail(SNN_E_INVALID, "engine node %u: unknown kind %u", n, nd.op);
    }
  }
  return SNN_OK;
}

}  // namespace

// Host images reach the device on the engine's copy stream, into the input
// buffer the previous forward is not reading (two buffers, alternating), so
// the copy of one call overlaps the forward of the previous one; each buffer
// has its own captured graph.
struct snn_engine {
  SnnEngineHeader h;
  std::vector<SnnEngineTensor> tensors;
  std::vector<SnnEngineNode> nodes;
  std::vector<void*> tptr;     // device address of every tensor
  uint8_t* arena = nullptr;    // tensors
  uint8_t* dblob = nullptr;    // parameters
  void* in_buf[2] = {nullptr, nullptr};   // input buffers (in_buf[0] is the arena's)
  int next = 0;
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t copied[2] = {nullptr, nullptr};
  cudaEvent_t buf_free[2] = {nullptr, nullptr};
  bool buf_used[2] = {false, false};
  int device = 0;
  cudaGraph_t graph[2] = {nullptr, nullptr};
  cudaGraphExec_t exec[2] = {nullptr, nullptr};
};

namespace {

int engine_node_loop(snn_engine* e, void* stream) {
  for (uint32_t n = 0; n < e->h.n_nodes; ++n) {
    const SnnEngineNode& nd = e->nodes[n];
    void* in0 = e->tptr[nd.in0];
    void* in1 = nd.in1 == kNoTensor ? nullptr : e->tptr[nd.in1];
    void* out = e->tptr[nd.out];
    auto P = [&](uint64_t off) { return reinterpret_cast<const float*>(e->dblob + off); };
    int st = SNN_OK;
    switch (nd.op) {
      case kOpStem:
        st = in1 ? snn_stem_forward_dual(&nd.desc, nd.i[0], static_cast<const float*>(in0), P(nd.p0),
                                         P(nd.p1), P(nd.p2), out, in1, stream)
                 : snn_stem_forward(&nd.desc, nd.i[0], static_cast<const float*>(in0), P(nd.p0),
                                    P(nd.p1), P(nd.p2), out, stream);
        break;
      case kOpConv:
        st = in1 ? snn_conv_forward_res(&nd.desc, in0, e->dblob + nd.p0, nullptr, P(nd.p1), P(nd.p2), in1,
                                        out, stream)
                 : snn_conv_forward(&nd.desc, in0, e->dblob + nd.p0, nullptr, P(nd.p1), P(nd.p2), out,
                                    stream);
        break;
      case kOpHead:
        st = snn_head_forward(nd.i[0], nd.i[1], nd.i[2], nd.i[3], nd.i[4], in0, P(nd.p0), P(nd.p1),
                              static_cast<float*>(out), stream);
        break;
      case kOpAddLif:
        st = snn_add_lif_forward(&nd.desc, in0, in1, nullptr, out, stream);
        break;
      case kOpMaxPoolLif:
        st = snn_maxpool_lif_forward(&nd.desc, in0, nullptr, out, stream);
        break;
      case kOpLif:
        st = snn_lif_forward(&nd.desc, in0, nullptr, out, stream);
        break;
      case kOpConvTsplit: {
        const uint32_t ws = static_cast<uint32_t>(nd.i[0]);
        st = snn_conv_forward_tsplit(&nd.desc, in0, e->dblob + nd.p0, nullptr, P(nd.p1), P(nd.p2), in1,
                                     out, e->tptr[ws], e->tensors[ws].bytes, stream);
        break;
      }
      case kOpAttn: {
        const snn_conv_desc& d = nd.desc;
        const void* vp = e->tptr[static_cast<uint32_t>(nd.i[0])];
        if (d.flags == SNN_FLAG_QKV_PACKED) {            // k and v: the next channel blocks
          const size_t cb = static_cast<size_t>(nd.i[2]) * nd.i[3] * 2;
          in1 = static_cast<char*>(in0) + cb;
          vp = static_cast<char*>(in0) + 2 * cb;
        }
        st = snn_spikformer_attn_forward(d.T, d.B, nd.i[1], nd.i[2], nd.i[3], d.tau2, d.tau,
                                         d.v_threshold, d.v_reset, d.flags, in0, in1, vp, nullptr,
                                         out, stream);
        break;
      }
      default:
        st = fail(SNN_E_INVALID, "engine node %u: unknown kind", n);
    }
    if (st) return st;
  }
  return SNN_OK;
}

bool is_host_pointer(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeUnregistered;
}

}  // namespace

extern "C" {

int snn_engine_check_file(const char* path, int32_t* n_nodes, int32_t* n_tensors) {
  SnnEngineHeader h;
  std::vector<SnnEngineTensor> t;
  std::vector<SnnEngineNode> n;
  std::vector<uint8_t> b;
  int st = parse_engine_file(path, &h, &t, &n, &b);
  if (st) return st;
  if (n_nodes) *n_nodes = static_cast<int32_t>(h.n_nodes);
  if (n_tensors) *n_tensors = static_cast<int32_t>(h.n_tensors);
  return SNN_OK;
}

void snn_engine_destroy(snn_engine* e) {
  if (!e) return;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(e->device);
  for (int k = 0; k < 2; ++k) {
    if (e->exec[k]) cudaGraphExecDestroy(e->exec[k]);
    if (e->graph[k]) cudaGraphDestroy(e->graph[k]);
    if (e->copied[k]) cudaEventDestroy(e->copied[k]);
    if (e->buf_free[k]) cudaEventDestroy(e->buf_free[k]);
  }
  if (e->copy_stream) cudaStreamDestroy(e->copy_stream);
  if (e->in_buf[1]) cudaFree(e->in_buf[1]);
  if (e->arena) cudaFree(e->arena);
  if (e->dblob) cudaFree(e->dblob);
  cudaSetDevice(cur);
  delete e;
}

int snn_engine_load(const char* path, snn_engine** out) {
  if (!out) return fail(SNN_E_INVALID, "engine out pointer is null");
  *out = nullptr;
  int st = ensure_init();
  if (st) return st;
  snn_engine* e = new snn_engine();
  std::vector<uint8_t> blob;
  st = parse_engine_file(path, &e->h, &e->tensors, &e->nodes, &blob);
  if (st) { delete e; return st; }
  cudaGetDevice(&e->device);
  uint64_t total = 0;
  std::vector<uint64_t> off(e->h.n_tensors);
  for (uint32_t t = 0; t < e->h.n_tensors; ++t) {
    off[t] = total;
    total += (e->tensors[t].bytes + 255) / 256 * 256;
  }
  cudaError_t ce = cudaMalloc(&e->arena, total);
  if (ce == cudaSuccess) ce = cudaMalloc(&e->in_buf[1], e->tensors[e->h.input].bytes);
  if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking);
  for (int k = 0; k < 2 && ce == cudaSuccess; ++k) {
    ce = cudaEventCreateWithFlags(&e->copied[k], cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&e->buf_free[k], cudaEventDisableTiming);
  }
  if (ce == cudaSuccess && e->h.blob_bytes) ce = cudaMalloc(&e->dblob, e->h.blob_bytes);
  if (ce == cudaSuccess && e->h.blob_bytes)
    ce = cudaMemcpy(e->dblob, blob.data(), e->h.blob_bytes, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) {
    snn_engine_destroy(e);
    return fail(SNN_E_CUDA, "engine device memory: %s", cudaGetErrorString(ce));
  }
  e->tptr.resize(e->h.n_tensors);
  for (uint32_t t = 0; t < e->h.n_tensors; ++t) e->tptr[t] = e->arena + off[t];
  e->in_buf[0] = e->tptr[e->h.input];
  *out = e;
  return SNN_OK;
}

int snn_engine_io(const snn_engine* e, int32_t* T, int32_t* B, size_t* image_bytes, size_t* logit_bytes) {
  if (!e) return fail(SNN_E_INVALID, "engine is null");
  if (T) *T = static_cast<int32_t>(e->h.T);
  if (B) *B = static_cast<int32_t>(e->h.B);
  if (image_bytes) *image_bytes = e->tensors[e->h.input].bytes;
  if (logit_bytes) *logit_bytes = e->tensors[e->h.output].bytes;
  return SNN_OK;
}

int snn_engine_capture(snn_engine* e, void* stream) {
  if (!e) return fail(SNN_E_INVALID, "engine is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!s) return fail(SNN_E_INVALID, "capture needs a non-default stream");
  for (int k = 0; k < 2; ++k) {
    if (e->exec[k]) { cudaGraphExecDestroy(e->exec[k]); e->exec[k] = nullptr; }
    if (e->graph[k]) { cudaGraphDestroy(e->graph[k]); e->graph[k] = nullptr; }
  }
  for (int k = 0; k < 2; ++k) {        // one graph per input buffer
    e->tptr[e->h.input] = e->in_buf[k];
    cudaError_t ce = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (ce != cudaSuccess) {
      e->tptr[e->h.input] = e->in_buf[0];
      return fail(SNN_E_CUDA, "begin capture: %s", cudaGetErrorString(ce));
    }
    int st = engine_node_loop(e, stream);
    cudaGraph_t g = nullptr;
    ce = cudaStreamEndCapture(s, &g);
    e->tptr[e->h.input] = e->in_buf[0];
    if (st) { if (g) cudaGraphDestroy(g); return st; }
    if (ce != cudaSuccess) return fail(SNN_E_CUDA, "end capture: %s", cudaGetErrorString(ce));
    ce = cudaGraphInstantiate(&e->exec[k], g, 0);
    if (ce != cudaSuccess) {
      cudaGraphDestroy(g);
      return fail(SNN_E_CUDA, "instantiate: %s", cudaGetErrorString(ce));
    }
    e->graph[k] = g;
  }
  return SNN_OK;
}

int snn_engine_run(snn_engine* e, const float* images, float* logits, void* stream) {
  if (!e) return fail(SNN_E_INVALID, "engine is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t ce = cudaSuccess;
  const int k = e->next;
  e->next ^= 1;
  void* din = e->in_buf[k];
  void* dout = e->tptr[e->h.output];
  if (images) {
    // Into buffer k on the copy stream, once the forward that last read it
    // is done; device images (which work on `stream` may still be writing)
    // and a first use also wait for everything issued on `stream` so far.
    const bool host = is_host_pointer(images);
    ce = e->buf_used[k] ? cudaStreamWaitEvent(e->copy_stream, e->buf_free[k], 0) : cudaSuccess;
    if (ce == cudaSuccess && (!host || !e->buf_used[k])) {
      ce = cudaEventRecord(e->copied[k], s);
      if (ce == cudaSuccess) ce = cudaStreamWaitEvent(e->copy_stream, e->copied[k], 0);
    }
    if (ce == cudaSuccess)
      ce = cudaMemcpyAsync(din, images, e->tensors[e->h.input].bytes,
                           host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, e->copy_stream);
    if (ce == cudaSuccess) ce = cudaEventRecord(e->copied[k], e->copy_stream);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(s, e->copied[k], 0);
    if (ce != cudaSuccess) return fail(SNN_E_CUDA, "images copy: %s", cudaGetErrorString(ce));
  } else if (din != e->in_buf[0]) {
    // No new images: the forward reads the engine's own input tensor.
    e->next = k;
    din = e->in_buf[0];
  }
  const int g = din == e->in_buf[0] ? 0 : 1;
  if (e->exec[g]) {
    ce = cudaGraphLaunch(e->exec[g], s);
    if (ce != cudaSuccess) return fail(SNN_E_CUDA, "graph launch: %s", cudaGetErrorString(ce));
  } else {
    e->tptr[e->h.input] = din;
    int st = engine_node_loop(e, stream);
    e->tptr[e->h.input] = e->in_buf[0];
    if (st) return st;
  }
  ce = cudaEventRecord(e->buf_free[g], s);
  if (ce != cudaSuccess) return fail(SNN_E_CUDA, "event: %s", cudaGetErrorString(ce));
  e->buf_used[g] = true;
  if (logits && logits != dout) {
    ce = cudaMemcpyAsync(logits, dout, e->tensors[e->h.output].bytes,
                         is_host_pointer(logits) ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s);
    if (ce != cudaSuccess) return fail(SNN_E_CUDA, "logits copy: %s", cudaGetErrorString(ce));
  }
  return SNN_OK;
}

}  // extern "C"
