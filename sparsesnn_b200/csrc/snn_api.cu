// C ABI of libsnnb200.so: descriptor validation, tensor-map construction,
// launches of the fused sparse layer, the dense stem and the classifier head.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <utility>

#include "../../include/snn_b200.h"
#include "snn_conv.cuh"
#include "snn_conv_halo.cuh"
#include "snn_conv_halo4.cuh"
#include "snn_conv_halo_stream.cuh"
#include "snn_glue.cuh"
#include "snn_attn.cuh"

namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

__device__ unsigned g_device_err = 0;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_init_mu;
bool g_inited = false;
int g_num_sms = 148;
int g_init_status = SNN_E_NO_DEVICE;

using ConvKernel = void (*)(const snn::ConvParams);

template <int MODE, int TC>
ConvKernel conv_kernel_fn_rm(int rm) {
  switch (rm) {
    case snn::kResAddAfter: return snn::fused_sparse_conv_lif_kernel<MODE, snn::kResAddAfter, TC>;
    case snn::kResAddBefore: return snn::fused_sparse_conv_lif_kernel<MODE, snn::kResAddBefore, TC>;
    case snn::kResTwoNeuron: return snn::fused_sparse_conv_lif_kernel<MODE, snn::kResTwoNeuron, TC>;
    default: return snn::fused_sparse_conv_lif_kernel<MODE, snn::kResNone, TC>;
  }
}
// Dense weights (two weight tiles per activation k-block): spiking neurons,
// no residual or the SEW add.
template <int MODE, int TC>
ConvKernel conv_dense_fn_rm(int rm) {
  return rm == snn::kResAddAfter
             ? snn::fused_sparse_conv_lif_kernel<MODE, snn::kResAddAfter, TC, false, 2>
             : snn::fused_sparse_conv_lif_kernel<MODE, snn::kResNone, TC, false, 2>;
}
template <int TC>
ConvKernel conv_kernel_fn_tc(int mode, int rm, bool dense) {
  if (dense) {
    switch (mode) {
      case snn::kModeLifHalf: return conv_dense_fn_rm<snn::kModeLifHalf, TC>(rm);
      case snn::kModeLifDiv: return conv_dense_fn_rm<snn::kModeLifDiv, TC>(rm);
      default: return conv_dense_fn_rm<snn::kModeIf, TC>(rm);
    }
  }
  switch (mode) {
    case snn::kModeLifHalf: return conv_kernel_fn_rm<snn::kModeLifHalf, TC>(rm);
    case snn::kModeLifDiv: return conv_kernel_fn_rm<snn::kModeLifDiv, TC>(rm);
    case snn::kModeIf: return conv_kernel_fn_rm<snn::kModeIf, TC>(rm);
    case snn::kModeBnF16:
      return rm == snn::kResAddAfter
                 ? snn::fused_sparse_conv_lif_kernel<snn::kModeBnF16, snn::kResAddAfter, TC>
                 : snn::fused_sparse_conv_lif_kernel<snn::kModeBnF16, snn::kResNone, TC>;
    default: return snn::fused_sparse_conv_lif_kernel<snn::kModeNone, snn::kResNone, TC>;
  }
}

// tc = timesteps per accumulator (2 or 4, see snn::GenCfg); rm = snn::ResMode.
ConvKernel conv_kernel_fn(int mode, int rm, int tc, bool dense = false) {
  return tc == 4 ? conv_kernel_fn_tc<4>(mode, rm, dense) : conv_kernel_fn_tc<2>(mode, rm, dense);
}
int conv_smem_bytes(int tc, bool dense) {
  if (dense) return tc == 4 ? snn::GenCfg<4, false, 2>::kSmemBytes : snn::GenCfg<2, false, 2>::kSmemBytes;
  return tc == 4 ? snn::GenCfg<4>::kSmemBytes : snn::GenCfg<2>::kSmemBytes;
}
// CTA-pair variant (TC = 4; spiking modes with no residual or the SEW add).
ConvKernel conv_pair_kernel_fn(int mode, int rm) {
  const bool res = rm == snn::kResAddAfter;
  switch (mode) {
    case snn::kModeLifHalf:
      return res ? snn::fused_sparse_conv_lif_kernel<snn::kModeLifHalf, snn::kResAddAfter, 4, true>
                 : snn::fused_sparse_conv_lif_kernel<snn::kModeLifHalf, snn::kResNone, 4, true>;
    case snn::kModeLifDiv:
      return res ? snn::fused_sparse_conv_lif_kernel<snn::kModeLifDiv, snn::kResAddAfter, 4, true>
                 : snn::fused_sparse_conv_lif_kernel<snn::kModeLifDiv, snn::kResNone, 4, true>;
    default:
      return res ? snn::fused_sparse_conv_lif_kernel<snn::kModeIf, snn::kResAddAfter, 4, true>
                 : snn::fused_sparse_conv_lif_kernel<snn::kModeIf, snn::kResNone, 4, true>;
  }
}

using HaloKernel = void (*)(const snn::HaloParams);

template <int BN, bool M64>
HaloKernel halo_kernel_fn_bn(int mode, bool res) {
  switch (mode * 2 + (res ? 1 : 0)) {
    case 0: return snn::fused_sparse_conv_halo_kernel<snn::kModeLifHalf, false, BN, 3, M64>;
    case 1: return snn::fused_sparse_conv_halo_kernel<snn::kModeLifHalf, true, BN, 3, M64>;
    case 2: return snn::fused_sparse_conv_halo_kernel<snn::kModeLifDiv, false, BN, 3, M64>;
    case 3: return snn::fused_sparse_conv_halo_kernel<snn::kModeLifDiv, true, BN, 3, M64>;
    case 4: return snn::fused_sparse_conv_halo_kernel<snn::kModeIf, false, BN, 3, M64>;
    case 5: return snn::fused_sparse_conv_halo_kernel<snn::kModeIf, true, BN, 3, M64>;
    default: return snn::fused_sparse_conv_halo_kernel<snn::kModeNone, false, BN, 3, M64>;
  }
}

// bn = 128 with m64 selects the M = 64 MMA path (layers of at most 64 channels).
HaloKernel halo4_kernel_fn(int mode, bool res) {
  if (mode == snn::kModeBnF16)
    return res ? snn::fused_sparse_conv_halo4_kernel<snn::kModeBnF16, true>
               : snn::fused_sparse_conv_halo4_kernel<snn::kModeBnF16, false>;
  switch (mode * 2 + (res ? 1 : 0)) {
    case 0: return snn::fused_sparse_conv_halo4_kernel<snn::kModeLifHalf, false>;
    case 1: return snn::fused_sparse_conv_halo4_kernel<snn::kModeLifHalf, true>;
    case 2: return snn::fused_sparse_conv_halo4_kernel<snn::kModeLifDiv, false>;
    case 3: return snn::fused_sparse_conv_halo4_kernel<snn::kModeLifDiv, true>;
    case 4: return snn::fused_sparse_conv_halo4_kernel<snn::kModeIf, false>;
    default: return snn::fused_sparse_conv_halo4_kernel<snn::kModeIf, true>;
  }
}

HaloKernel halo_kernel_fn(int bn, bool m64, int mode, bool res) {
  if (bn == 128) return m64 ? halo_kernel_fn_bn<128, true>(mode, res)
                            : halo_kernel_fn_bn<128, false>(mode, res);
  return halo_kernel_fn_bn<64, false>(mode, res);
}

using HsKernel = void (*)(const snn::ConvParams);

template <bool SMALL>
HsKernel hs_kernel_fn_t(int mode, bool res) {
  switch (mode * 2 + (res ? 1 : 0)) {
    case 0: return snn::fused_sparse_conv_halo_stream_kernel<snn::kModeLifHalf, false, SMALL>;
    case 1: return snn::fused_sparse_conv_halo_stream_kernel<snn::kModeLifHalf, true, SMALL>;
    case 2: return snn::fused_sparse_conv_halo_stream_kernel<snn::kModeLifDiv, false, SMALL>;
    case 3: return snn::fused_sparse_conv_halo_stream_kernel<snn::kModeLifDiv, true, SMALL>;
    case 4: return snn::fused_sparse_conv_halo_stream_kernel<snn::kModeIf, false, SMALL>;
    case 5: return snn::fused_sparse_conv_halo_stream_kernel<snn::kModeIf, true, SMALL>;
    default: return snn::fused_sparse_conv_halo_stream_kernel<snn::kModeNone, false, SMALL>;
  }
}
HsKernel hs_kernel_fn(int mode, bool res, bool small) {
  return small ? hs_kernel_fn_t<true>(mode, res) : hs_kernel_fn_t<false>(mode, res);
}

using StemKernel = void (*)(const snn::StemParams);

StemKernel stem_tc_fn(int cin, int mode) {
  if (cin == 3) {
    if (mode == snn::kModeLifHalf) return snn::stem_tc_kernel<3, snn::kModeLifHalf>;
    if (mode == snn::kModeLifDiv) return snn::stem_tc_kernel<3, snn::kModeLifDiv>;
    return snn::stem_tc_kernel<3, snn::kModeIf>;
  }
  if (mode == snn::kModeLifHalf) return snn::stem_tc_kernel<1, snn::kModeLifHalf>;
  if (mode == snn::kModeLifDiv) return snn::stem_tc_kernel<1, snn::kModeLifDiv>;
  return snn::stem_tc_kernel<1, snn::kModeIf>;
}
constexpr int kStemTcSmemMax = 96 * 1024;

// mode: the neuron (kModeNone: fp16 BN output); dual: fp16 BN output plus
// the spikes of `mode`'s neuron on it.
StemKernel stem_tcg_fn(int mode, bool dual = false) {
  if (dual) {
    switch (mode) {
      case snn::kModeLifHalf: return snn::stem_tc_gen_kernel<snn::kModeLifHalf, true>;
      case snn::kModeLifDiv: return snn::stem_tc_gen_kernel<snn::kModeLifDiv, true>;
      default: return snn::stem_tc_gen_kernel<snn::kModeIf, true>;
    }
  }
  switch (mode) {
    case snn::kModeLifHalf: return snn::stem_tc_gen_kernel<snn::kModeLifHalf, false>;
    case snn::kModeLifDiv: return snn::stem_tc_gen_kernel<snn::kModeLifDiv, false>;
    case snn::kModeIf: return snn::stem_tc_gen_kernel<snn::kModeIf, false>;
    default: return snn::stem_tc_gen_kernel<snn::kModeNone, false>;
  }
}

constexpr int kSmemLimit = 232448;          // opt-in dynamic smem per block on sm_100

// Launches with programmatic stream serialization: the kernel may be
// scheduled while its predecessor in the stream drains (the kernels run their
// prologue on constant data, then griddepcontrol.wait before touching stream
// data).  Returns the launch status.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
// Same for a kernel launched as 2-CTA clusters (grid.x even).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_pair(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
constexpr int kHaloMaxWeightBytes = 160 * 1024;

int ensure_init() {
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (g_inited) return g_init_status;
  g_inited = true;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return g_init_status = fail(SNN_E_NO_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) return g_init_status = fail(SNN_E_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
  if (prop.major != 10 || prop.minor != 0)
    return g_init_status = fail(SNN_E_NO_DEVICE, "device sm_%d%d is not sm_100", prop.major, prop.minor);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return g_init_status = fail(SNN_E_CUDA, "cuTensorMapEncodeTiled unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  g_num_sms = prop.multiProcessorCount;
  for (int mode = 0; mode < 4; ++mode) {
    for (int res = 0; res < (mode == snn::kModeNone ? 1 : 2); ++res) {
      for (int tc : {2, 4}) {
        // res == 1 covers every residual epilogue of the general kernel.
        for (int rm = res; rm <= (res ? snn::kResTwoNeuron : 0); ++rm) {
          e = cudaFuncSetAttribute(conv_kernel_fn(mode, rm, tc),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   tc == 4 ? snn::GenCfg<4>::kSmemBytes : snn::GenCfg<2>::kSmemBytes);
          if (e != cudaSuccess)
            return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
        }
      }
      for (int v = 0; v < 3; ++v) {
        e = cudaFuncSetAttribute(halo_kernel_fn(v ? 128 : 64, v == 2, mode, res != 0),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess)
          return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
      }
      if (mode != snn::kModeNone) {
        e = cudaFuncSetAttribute(halo4_kernel_fn(mode, res != 0),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess)
          return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
      }
      if (mode != snn::kModeNone && res == 0) {
        for (int cin : {1, 3}) {
          e = cudaFuncSetAttribute(stem_tc_fn(cin, mode),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kStemTcSmemMax);
          if (e != cudaSuccess)
            return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
        }
      }
      for (int small = 0; small < 2; ++small) {
        e = cudaFuncSetAttribute(hs_kernel_fn(mode, res != 0, small != 0),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, snn::kHsSmemBytes);
        if (e != cudaSuccess)
          return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
      }
    }
  }
  for (int res = 0; res < 2 && e == cudaSuccess; ++res)
    e = cudaFuncSetAttribute(halo4_kernel_fn(snn::kModeBnF16, res != 0),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  for (int tc : {2, 4}) {
    // fp16 BN output, plain and plus a residual; dense-weight spiking layers.
    for (int rm : {snn::kResNone, snn::kResAddAfter}) {
      e = cudaFuncSetAttribute(conv_kernel_fn(snn::kModeBnF16, rm, tc),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, conv_smem_bytes(tc, false));
      for (int mode = 0; mode < 3 && e == cudaSuccess; ++mode)
        e = cudaFuncSetAttribute(conv_kernel_fn(mode, rm, tc, true),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, conv_smem_bytes(tc, true));
      if (e != cudaSuccess)
        return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
    }
  }
  for (int mode = 0; mode < 4 && e == cudaSuccess; ++mode)
    for (int dual = 0; dual < 2 && e == cudaSuccess; ++dual)
      e = cudaFuncSetAttribute(stem_tcg_fn(mode, dual != 0), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               snn::stem_tcg_smem_max());
  if (e != cudaSuccess)
    return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
  e = cudaFuncSetAttribute(snn::spikformer_attn_lif_kernel<32>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, snn::AttnCfg<32>::kSmemBytes);
  for (int mode = 0; mode < 3 && e == cudaSuccess; ++mode)
    for (int rm = 0; rm < 2 && e == cudaSuccess; ++rm)
      e = cudaFuncSetAttribute(conv_pair_kernel_fn(mode, rm), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               snn::GenCfg<4, true>::kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(snn::spikformer_attn_lif_kernel<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, snn::AttnCfg<64>::kSmemBytes);
  if (e != cudaSuccess)
    return g_init_status = fail(SNN_E_CUDA, "smem attribute: %s", cudaGetErrorString(e));
  return g_init_status = SNN_OK;
}

struct Geometry {
  int OH, OW, K, Fpad, n_kb, cin_blocks;
  int kdup;    // compressed weight tiles per activation k-block (2: dense weights)
  int Kw;      // weight columns of the packed blob, K * kdup
};

int check_desc(const snn_conv_desc* d, Geometry* g) {
  if (!d) return fail(SNN_E_INVALID, "null descriptor");
  if (d->T < 1 || d->B < 1 || d->H < 1 || d->W < 1 || d->Cout < 1 || d->KH < 1 || d->KW < 1)
    return fail(SNN_E_INVALID, "non-positive dimension");
  // Input channels in 64-channel k-blocks; a partial last block (Cin a
  // multiple of 8, 16-byte pixel rows) reads zeros past Cin (TMA zero fill)
  // and its weight columns are zero.
  if (d->Cin < 8 || d->Cin % 8)
    return fail(SNN_E_INVALID, "Cin=%d must be a positive multiple of 8", d->Cin);
  if (d->Cout % 8) return fail(SNN_E_INVALID, "Cout=%d must be a multiple of 8", d->Cout);
  if (d->stride != 1 && d->stride != 2) return fail(SNN_E_INVALID, "stride must be 1 or 2");
  if (d->pad < 0 || d->pad >= d->KH || d->pad >= d->KW) return fail(SNN_E_INVALID, "bad pad");
  if (d->stride == 2 && ((d->H & 1) || (d->W & 1)))
    return fail(SNN_E_INVALID, "stride-2 layers need even H and W");
  if (d->neuron < SNN_NEURON_LIF || d->neuron > SNN_NEURON_NONE_F16)
    return fail(SNN_E_INVALID, "bad neuron kind");
  if (d->neuron == SNN_NEURON_LIF && !(d->tau > 0.f)) return fail(SNN_E_INVALID, "tau must be > 0");
  g->OH = (d->H + 2 * d->pad - d->KH) / d->stride + 1;
  g->OW = (d->W + 2 * d->pad - d->KW) / d->stride + 1;
  if (g->OH < 1 || g->OW < 1) return fail(SNN_E_INVALID, "empty output");
  g->cin_blocks = (d->Cin + snn::kKB - 1) / snn::kKB;
  g->K = d->KH * d->KW * g->cin_blocks * snn::kKB;       // GEMM K (input channels padded)
  g->Fpad = (d->Cout + snn::kBM - 1) / snn::kBM * snn::kBM;
  g->n_kb = d->KH * d->KW * g->cin_blocks;
  g->kdup = (d->flags & SNN_FLAG_DENSE) ? 2 : 1;
  g->Kw = g->K * g->kdup;
  if (g->Kw / 32 > snn::kMaxMetaCols)
    return fail(SNN_E_INVALID, "K=%d exceeds the %d supported%s", g->K, snn::kMaxMetaCols * 32 / g->kdup,
                g->kdup > 1 ? " for dense weights" : "");
  if ((long long)d->T * d->B > 0x7fffffffLL) return fail(SNN_E_INVALID, "T*B too large");
  if ((long long)d->B * g->OH * g->OW > 0x7fffffffLL)
    return fail(SNN_E_INVALID, "B*OH*OW too large");
  return SNN_OK;
}

size_t meta_offset(const Geometry& g) {
  size_t vbytes = static_cast<size_t>(g.Fpad) * (g.Kw / 2) * 2;
  return (vbytes + 255) & ~static_cast<size_t>(255);
}

int encode(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swz,
           CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT16) {
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), dims,
                        strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SNN_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SNN_OK;
}

// Which kernel serves a descriptor (see the SNN_VARIANT_* values).
// Pixels per tile of the general kernel: up to 64 pixels of one timestep --
// a run of one output row, whole rows of one image, or whole images.
void general_tile(const Geometry& g, int B, int* tw, int* th, int* tn) {
  if (g.OW >= snn::kBN) { *tw = snn::kBN; *th = 1; *tn = 1; }
  else if (snn::kBN % g.OW == 0 && g.OH * g.OW >= snn::kBN) { *tw = g.OW; *th = snn::kBN / g.OW; *tn = 1; }
  else if (g.OW > 4 && g.OH > 4) {
    // Other widths (56, 28, 14, 7, ...): 8 x 8-pixel tiles, whose 64-pixel
    // boxes let the four-timestep N = 256 MMAs run (ragged edges read zero
    // fill and are not stored) -- measured faster than whole-row tiles of
    // fewer than 64 pixels, which fall back to per-timestep N = 64 MMAs.
    *tw = 8; *th = 8; *tn = 1;
  }
  else { *tw = g.OW; *th = g.OH; *tn = std::max(1, std::min(B, snn::kBN / (g.OH * g.OW))); }
}

int select_variant(const snn_conv_desc* d, const Geometry& g) {
  if (d->flags & SNN_FLAG_FORCE_GENERIC) return SNN_VARIANT_GENERIC;
  // Dense weights run in the general kernel only; the fp16 BN output also in
  // the four-timestep halo kernel (<= 64 channels, stride-1 3x3, below).
  if (d->flags & SNN_FLAG_DENSE) return SNN_VARIANT_GENERIC;
  if (d->neuron == SNN_NEURON_NONE_F16 &&
      !(d->Cout <= 64 && d->stride == 1 && d->KH == 3 && d->KW == 3 && d->pad == 1 && g.OW >= 8 &&
        g.OH >= 8 && g.n_kb * snn::kABytes <= kHaloMaxWeightBytes))
    return SNN_VARIANT_GENERIC;
  // Only the general kernel has the Add-before-neuron and two-neuron epilogues.
  if (d->res_mode != SNN_RES_ADD_AFTER) return SNN_VARIANT_GENERIC;
  const bool s1_3x3 = d->stride == 1 && d->KH == 3 && d->KW == 3 && d->pad == 1;
  if (!s1_3x3) return SNN_VARIANT_GENERIC;
  const int a_bytes = g.n_kb * snn::kABytes;
  if (a_bytes <= kHaloMaxWeightBytes && g.OH >= 8) return SNN_VARIANT_HALO_RESIDENT;
  // Streamed weights: the streaming halo kernel loads each tile's input halo
  // once for all nine taps and T <= 4 timesteps (the general kernel loads a
  // box per tap), measured faster on 8x8 and 12x12 images.
  if (((g.OH >= 8 && g.OW >= 8) || (g.OH == 4 && g.OW == 4)) && d->T <= snn::kHsMaxT)
    return SNN_VARIANT_HALO_STREAM;
  return SNN_VARIANT_GENERIC;
}

// rm: snn::ResMode of the call (kResNone when residual is null).
int launch_conv(const snn_conv_desc* d, const void* data, const void* weight, float* state,
                float* state2, const float* scale, const float* bias, const void* residual,
                int rm, void* out, void* stream) {
  int st = ensure_init();
  if (st) return st;
  Geometry g;
  if ((st = check_desc(d, &g))) return st;
  if (!data || !weight || !scale || !bias || !out) return fail(SNN_E_INVALID, "null tensor pointer");
  if ((d->flags & (SNN_FLAG_READ_STATE | SNN_FLAG_WRITE_STATE)) && !state)
    return fail(SNN_E_INVALID, "state flags set but state is null");
  if (d->neuron == SNN_NEURON_NONE && residual)
    return fail(SNN_E_INVALID, "residual needs a neuron (or the fp16 BN output)");
  if (d->neuron == SNN_NEURON_NONE_F16 && residual && rm != snn::kResAddAfter)
    return fail(SNN_E_INVALID, "fp16 BN output takes only the ADD_AFTER residual");
  if (g.kdup > 1 && (d->neuron >= SNN_NEURON_NONE || (residual && rm != snn::kResAddAfter)))
    return fail(SNN_E_INVALID, "dense weights: spiking neuron, no residual or the SEW add");
  if (rm == snn::kResTwoNeuron) {
    if ((d->flags & (SNN_FLAG_READ_STATE | SNN_FLAG_WRITE_STATE)) && !state2)
      return fail(SNN_E_INVALID, "state flags set but state2 is null");
    if (d->neuron2 != SNN_NEURON_LIF && d->neuron2 != SNN_NEURON_IF)
      return fail(SNN_E_INVALID, "neuron2 must be LIF or IF");
    if (d->neuron2 == SNN_NEURON_LIF && !(d->tau2 > 0.0f))
      return fail(SNN_E_INVALID, "tau2 must be positive");
  }
  if ((reinterpret_cast<uintptr_t>(data) | reinterpret_cast<uintptr_t>(weight) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) & 15)
    return fail(SNN_E_INVALID, "data, weight, out and residual must be 16-byte aligned");

  snn::ConvParams p;
  memset(&p, 0, sizeof(p));
  const char* wbytes = static_cast<const char*>(weight);
  {  // compressed weights [Fpad][Kw/2]
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(g.Kw / 2), static_cast<cuuint64_t>(g.Fpad)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(g.Kw / 2) * 2};
    cuuint32_t box[2] = {snn::kKB / 2, snn::kBM};
    if ((st = encode(&p.tmap_a, 2, wbytes, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
  }
  // Tile geometry in output coordinates: a tile is up to 64 pixels of one
  // timestep -- a run of one output row, whole rows of one image, or whole
  // images.
  int tw, th, tn;
  general_tile(g, d->B, &tw, &th, &tn);
  p.tw = tw; p.th = th; p.tn = tn;
  p.tiles_w = (g.OW + tw - 1) / tw;
  p.tiles_h = (g.OH + th - 1) / th;
  const int tiles_n = (d->B + tn - 1) / tn;
  const long long n_px = static_cast<long long>(p.tiles_w) * p.tiles_h * tiles_n;
  if (n_px > 0x7fffffffLL) return fail(SNN_E_INVALID, "too many pixel tiles");
  p.n_px_tiles = static_cast<int>(n_px);
  p.n_m = g.Fpad / snn::kBM;
  p.box_bytes = tw * th * tn * snn::kKB * 2;
  // Timesteps per accumulator of the general kernel: all four (N = 256 MMAs,
  // one accumulator) for 64-pixel tiles when T is a multiple of 4 -- the
  // wider MMAs win even though a CTA's next tile then waits for the
  // epilogue to drain the accumulator -- else two (N = 128, double-buffered).
  const int tc = (d->T % 4 == 0 && p.box_bytes == snn::kBBytes) ? 4 : 2;
  // CTA pairs (on request) for those layers when the 128-channel tiles come
  // in pairs: each CTA loads half of the four-timestep activation box.  3x3
  // only (the 1x1 downsamples measured slower).
  const bool pair = (d->flags & SNN_FLAG_CTA_PAIR) && tc == 4 && p.n_m % 2 == 0 &&
                    d->neuron < SNN_NEURON_NONE && g.kdup == 1 && d->KH * d->KW > 1 &&
                    (rm == snn::kResNone || rm == snn::kResAddAfter);
  const cuuint32_t box5[5] = {static_cast<cuuint32_t>(snn::kKB), static_cast<cuuint32_t>(tw),
                              static_cast<cuuint32_t>(th), static_cast<cuuint32_t>(tn),
                              static_cast<cuuint32_t>(pair ? tc / 2 : tc)};
  {
    const size_t C = d->Cin, W = d->W, H = d->H, B = d->B;
    const char* base = static_cast<const char*>(data);
    const int nmaps = d->stride == 2 ? 4 : 1;
    for (int m = 0; m < nmaps; ++m) {
      const int hp = m >> 1, wp = m & 1;
      cuuint64_t dims[5], strides[4];
      const char* b = base;
      if (d->stride == 1) {
        dims[1] = W; dims[2] = H;
        strides[0] = C * 2; strides[1] = W * C * 2;
      } else {
        dims[1] = (W - wp + 1) / 2; dims[2] = (H - hp + 1) / 2;
        strides[0] = 2 * C * 2; strides[1] = 2 * W * C * 2;
        b = base + (hp * W + wp) * C * 2;
      }
      dims[0] = C; dims[3] = B; dims[4] = static_cast<cuuint64_t>(d->T);
      strides[2] = H * W * C * 2; strides[3] = B * H * W * C * 2;
      if ((st = encode(&p.tmap_b[m], 5, b, dims, strides, box5, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    }
  }
  // fp16 output (spikes, spikes + residual, or the fp16 BN output) or fp32 BN output.
  const bool spikes = d->neuron != SNN_NEURON_NONE;
  if (spikes) p.out = static_cast<__half*>(out);
  else p.out_f32 = static_cast<float*>(out);
  p.residual = static_cast<const __half*>(residual);
  p.meta = reinterpret_cast<const uint32_t*>(wbytes + meta_offset(g));
  p.scale = scale; p.bias = bias; p.state = state; p.state2 = state2;
  unsigned* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_device_err) != cudaSuccess)
    return fail(SNN_E_CUDA, "error word address");
  p.err = err;
  p.F = d->Cout; p.KW = d->KW; p.stride = d->stride; p.pad = d->pad;
  p.n_kb = g.n_kb; p.cin_blocks = g.cin_blocks;
  p.B = d->B; p.OH = g.OH; p.OW = g.OW; p.T = d->T;
  p.flags = d->flags;
  p.tau = d->tau;
  // Reference computes (1.0 - 1.0/tau) in double, then float32 (models/neurons.py:125).
  p.decay = d->neuron == SNN_NEURON_LIF
                ? static_cast<float>(1.0 - 1.0 / static_cast<double>(d->tau)) : 1.0f;
  p.inv_tau = 0.0f;
  p.v_th = d->v_threshold; p.v_reset = d->v_reset;
  if (rm == snn::kResTwoNeuron) {
    p.n2_lif = d->neuron2 == SNN_NEURON_LIF;
    p.tau2 = p.n2_lif ? d->tau2 : 1.0f;
    p.decay2 = p.n2_lif ? static_cast<float>(1.0 - 1.0 / static_cast<double>(d->tau2)) : 1.0f;
    p.v_th2 = d->v_threshold2; p.v_reset2 = d->v_reset2;
  }
  p.timeout_ns = 4000000000ull;   // SM cycles (~2 s at the highest clock)
  const int mode = d->neuron == SNN_NEURON_NONE ? snn::kModeNone
                   : d->neuron == SNN_NEURON_NONE_F16 ? snn::kModeBnF16
                   : d->neuron == SNN_NEURON_IF ? snn::kModeIf
                   : d->tau == 2.0f ? snn::kModeLifHalf : snn::kModeLifDiv;

  // Halo variant: stride-1 odd square kernels with "same" padding whose
  // 128-channel weight slice fits in shared memory and images tall enough
  // for 8-row tiles.
  const int a_bytes = g.n_kb * snn::kABytes;
  const int variant = select_variant(d, g);
  if (variant == SNN_VARIANT_HALO_RESIDENT) {
    snn::HaloParams hp;
    memset(&hp, 0, sizeof(hp));
    // Spiking layers with at most 64 output channels: one N = 256 MMA per
    // tap covers 8 x 8 pixels x 4 timesteps (fused_sparse_conv_halo4_kernel).
    if (d->Cout <= 64 && mode != snn::kModeNone && g.OW >= 8 && p.n_m == 1) {
      const int a4 = a_bytes / 2;                // the 64 real weight rows
      const int halo_w = 8 + d->KW - 1;
      const int halo_bytes = snn::kKB * 2 * halo_w * snn::kH4Ts * (8 + d->KH - 1);
      const int halo_stride = (halo_bytes + 1023) / 1024 * 1024;
      const int fixed = 1024 + 512 + a4 + 2 * snn::kH4OutBytes;
      const int stages = std::min(snn::kH4MaxStages, (kSmemLimit - fixed) / halo_stride);
      if (stages >= 2) {
        cuuint64_t wdims[3] = {static_cast<cuuint64_t>(snn::kKB / 2), static_cast<cuuint64_t>(g.Fpad),
                               static_cast<cuuint64_t>(g.n_kb)};
        cuuint64_t wstrides[2] = {static_cast<cuuint64_t>(g.K / 2) * 2,
                                  static_cast<cuuint64_t>(snn::kKB / 2) * 2};
        cuuint32_t wbox[3] = {snn::kKB / 2, 64, static_cast<cuuint32_t>(g.n_kb)};
        if ((st = encode(&p.tmap_a, 3, wbytes, wdims, wstrides, wbox, CU_TENSOR_MAP_SWIZZLE_64B)))
          return st;
        p.tw = 8; p.th = 8; p.tn = 1;
        p.tiles_w = (g.OW + 7) / 8;
        p.tiles_h = (g.OH + 7) / 8;
        p.n_px_tiles = p.tiles_w * p.tiles_h * d->B;
        // Activations seen as (C, W, T, H, B): one box holds a tile's halo
        // for four timesteps as [halo row][timestep][halo column].
        const size_t C = d->Cin, W = d->W, H = d->H, B = d->B;
        cuuint64_t dims[5] = {C, W, static_cast<cuuint64_t>(d->T), H, B};
        cuuint64_t strides[4] = {C * 2, B * H * W * C * 2, W * C * 2, H * W * C * 2};
        cuuint32_t box[5] = {static_cast<cuuint32_t>(snn::kKB), static_cast<cuuint32_t>(halo_w),
                             static_cast<cuuint32_t>(snn::kH4Ts), static_cast<cuuint32_t>(8 + d->KH - 1), 1};
        if ((st = encode(&p.tmap_b[0], 5, data, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)))
          return st;
        // Output (and SEW residual) seen as (F, OW, OH, B, T) with boxes of
        // 64 channels x 8 x 8 pixels x 4 timesteps; channels past F and
        // pixels or timesteps past the tensor are not stored (read as zero).
        {
          const size_t F = d->Cout, OW = g.OW, OH = g.OH;
          cuuint64_t odims[5] = {F, OW, OH, B, static_cast<cuuint64_t>(d->T)};
          cuuint64_t ostrides[4] = {F * 2, OW * F * 2, OH * OW * F * 2, B * OH * OW * F * 2};
          cuuint32_t obox[5] = {64, 8, 8, 1, static_cast<cuuint32_t>(snn::kH4Ts)};
          if ((st = encode(&p.tmap_b[1], 5, out, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_128B)))
            return st;
          if (residual &&
              (st = encode(&p.tmap_b[2], 5, residual, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_128B)))
            return st;
        }
        hp.KH = d->KH;
        hp.halo_w = halo_w;
        hp.halo_bytes = halo_bytes;
        hp.halo_stride = halo_stride;
        hp.halo_stages = stages;
        hp.a_bytes = a4;
        hp.c = p;
        const size_t smem = static_cast<size_t>(fixed) + static_cast<size_t>(stages) * halo_stride;
        const int grid = std::max(1, std::min(p.n_px_tiles, g_num_sms));
        cudaError_t e = launch_pdl(halo4_kernel_fn(mode, residual != nullptr), dim3(grid),
                                   dim3(snn::kH4Threads), smem, stream, hp);
        if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
        return SNN_OK;
      }
    }
  }
  if (variant == SNN_VARIANT_HALO_RESIDENT && mode != snn::kModeBnF16) {
    snn::HaloParams hp;
    memset(&hp, 0, sizeof(hp));
    const int bn = g.OH >= 16 ? 128 : 64;
    const bool m64 = bn == 128 && d->Cout <= 64;
    const int th_ = bn / 8;
    hp.KH = d->KH;
    hp.halo_w = 8 + d->KW - 1;
    hp.halo_bytes = hp.halo_w * (th_ + d->KH - 1) * snn::kKB * 2;
    hp.halo_stride = (hp.halo_bytes + 1023) / 1024 * 1024;
    // M = 64 keeps only the 64 real weight rows resident (box of 64 rows).
    hp.a_bytes = m64 ? a_bytes / 2 : a_bytes;
    {
      // The packed weights [Fpad][K/2] seen as [k-block][row][32 elements]:
      // one box delivers a CTA's whole slice in the k-block-major order the
      // MMA descriptors expect.
      cuuint64_t dims[3] = {static_cast<cuuint64_t>(snn::kKB / 2), static_cast<cuuint64_t>(g.Fpad),
                            static_cast<cuuint64_t>(g.n_kb)};
      cuuint64_t strides[2] = {static_cast<cuuint64_t>(g.K / 2) * 2, static_cast<cuuint64_t>(snn::kKB / 2) * 2};
      cuuint32_t box[3] = {snn::kKB / 2, static_cast<cuuint32_t>(m64 ? 64 : snn::kBM),
                           static_cast<cuuint32_t>(g.n_kb)};
      if (g.n_kb > 256) return fail(SNN_E_INVALID, "too many k-blocks for the resident weight box");
      if ((st = encode(&p.tmap_a, 3, wbytes, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
    }
    const int fixed = 1024 + 512 + (m64 ? snn::kHalo64XposeBytes : snn::kHaloXposeBytes) + hp.a_bytes;
    hp.halo_stages = std::min(snn::kHaloMaxStages, (kSmemLimit - fixed) / hp.halo_stride);
    if (hp.halo_stages >= 2) {
      p.tw = 8; p.th = th_; p.tn = 1;
      p.tiles_w = (g.OW + 7) / 8;
      p.tiles_h = (g.OH + th_ - 1) / th_;
      p.n_px_tiles = p.tiles_w * p.tiles_h * d->B;
      const size_t C = d->Cin, W = d->W, H = d->H, B = d->B;
      cuuint64_t dims[5] = {C, W, H, B, static_cast<cuuint64_t>(d->T)};
      cuuint64_t strides[4] = {C * 2, W * C * 2, H * W * C * 2, B * H * W * C * 2};
      cuuint32_t box[5] = {static_cast<cuuint32_t>(snn::kKB), static_cast<cuuint32_t>(hp.halo_w),
                           static_cast<cuuint32_t>(th_ + d->KH - 1), 1, 1};
      if ((st = encode(&p.tmap_b[0], 5, data, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
      if (!m64 && mode != snn::kModeNone) {
        // Spike output as (F, OW, OH, B, T): a warp stores {32 ch, 8 w, 4 h}
        // from its transpose tile (64-byte swizzle).
        const size_t F = d->Cout, OW = g.OW, OH = g.OH;
        cuuint64_t odims[5] = {F, OW, OH, B, static_cast<cuuint64_t>(d->T)};
        cuuint64_t ostrides[4] = {F * 2, OW * F * 2, OH * OW * F * 2, B * OH * OW * F * 2};
        cuuint32_t obox[5] = {32, 8, 4, 1, 1};
        if ((st = encode(&p.tmap_b[1], 5, out, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_64B)))
          return st;
      }
      hp.c = p;
      const size_t smem = static_cast<size_t>(fixed) + static_cast<size_t>(hp.halo_stages) * hp.halo_stride;
      const int per_m = std::max(1, std::min(p.n_px_tiles, g_num_sms / p.n_m));
      const long long grid = static_cast<long long>(per_m) * p.n_m;
      cudaError_t e = launch_pdl(halo_kernel_fn(bn, m64, mode, residual != nullptr),
                                 dim3(static_cast<unsigned>(grid)), dim3(snn::kHaloThreads), smem,
                                 stream, hp);
      if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
      return SNN_OK;
    }
  }
  // Streaming-weight halo variant: stride-1 3x3 "same" convs on images of
  // at least 8x8 whose weights do not fit in shared memory, T <= 4.
  if (variant == SNN_VARIANT_HALO_STREAM) {
    snn::ConvParams ph = p;
    // 4x4 images: a tile is 4 whole images, loaded as three column-shifted
    // boxes per input slice (the kernel's SMALL form).
    const bool small = g.OH == 4 && g.OW == 4;
    const size_t C = d->Cin, W = d->W, H = d->H, B = d->B;
    if (small) {
      ph.tw = 4; ph.th = 4; ph.tn = 4;
      ph.tiles_w = 1; ph.tiles_h = 1;
      ph.n_px_tiles = (d->B + 3) / 4;
      // Activations seen as (C, W, T, B, H): [halo row][image][timestep][4 columns].
      cuuint64_t dims[5] = {C, W, static_cast<cuuint64_t>(d->T), B, H};
      cuuint64_t strides[4] = {C * 2, B * H * W * C * 2, H * W * C * 2, W * C * 2};
      cuuint32_t box[5] = {static_cast<cuuint32_t>(snn::kKB), 4, static_cast<cuuint32_t>(d->T), 4, 6};
      if ((st = encode(&ph.tmap_b[0], 5, data, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
      // Weights as (Cpad/2 el of one tap, Fpad rows, kh, kw): one box = taps (0..2, kw).
      const size_t Cp = static_cast<size_t>(g.cin_blocks) * snn::kKB;
      cuuint64_t wd[4] = {Cp / 2, static_cast<cuuint64_t>(g.Fpad), 3, 3};
      cuuint64_t ws[3] = {static_cast<cuuint64_t>(g.K / 2) * 2, 3 * (Cp / 2) * 2, (Cp / 2) * 2};
      cuuint32_t wb[4] = {snn::kKB / 2, snn::kBM, 3, 1};
      if ((st = encode(&ph.tmap_b[1], 4, weight, wd, ws, wb, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
    } else {
      ph.tw = 8; ph.th = 8; ph.tn = 1;
      ph.tiles_w = (g.OW + 7) / 8;
      ph.tiles_h = (g.OH + 7) / 8;
      ph.n_px_tiles = ph.tiles_w * ph.tiles_h * d->B;
      // Activations seen as (C, W, T, H, B): one box holds a tile's halo for
      // all T timesteps as [halo row][timestep][halo column].
      cuuint64_t dims[5] = {C, W, static_cast<cuuint64_t>(d->T), H, B};
      cuuint64_t strides[4] = {C * 2, B * H * W * C * 2, W * C * 2, H * W * C * 2};
      cuuint32_t box[5] = {static_cast<cuuint32_t>(snn::kKB), 10, static_cast<cuuint32_t>(d->T), 10, 1};
      if ((st = encode(&ph.tmap_b[0], 5, data, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
      // weights as (Cpad/2 el of one tap, Fpad rows, 9 taps): one box = 3 taps x 128 rows
      const size_t Cp = static_cast<size_t>(g.cin_blocks) * snn::kKB;
      cuuint64_t wd[3] = {Cp / 2, static_cast<cuuint64_t>(g.Fpad), 9};
      cuuint64_t ws[2] = {static_cast<cuuint64_t>(g.K / 2) * 2, (Cp / 2) * 2};
      cuuint32_t wb[3] = {snn::kKB / 2, snn::kBM, 3};
      if ((st = encode(&ph.tmap_b[1], 3, weight, wd, ws, wb, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
    }
    if (spikes) {  // spikes as (F, OW, OH, B, T): a warp stores {32 ch, 8 w, 4 h} ({32, 4, 4, 2} SMALL)
      const size_t F = d->Cout, OW = g.OW, OH = g.OH;
      cuuint64_t odims[5] = {F, OW, OH, B, static_cast<cuuint64_t>(d->T)};
      cuuint64_t ostrides[4] = {F * 2, OW * F * 2, OH * OW * F * 2, B * OH * OW * F * 2};
      cuuint32_t obox[5] = {32, small ? 4u : 8u, 4, small ? 2u : 1u, 1};
      if ((st = encode(&ph.tmap_out, 5, out, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
      ph.tma_out = 1;
    }
    const int per_m = std::max(1, std::min(ph.n_px_tiles, g_num_sms / ph.n_m));
    const long long grid = static_cast<long long>(per_m) * ph.n_m;
    cudaError_t e = launch_pdl(hs_kernel_fn(mode, residual != nullptr, small),
                               dim3(static_cast<unsigned>(grid)), dim3(snn::kHaloThreads),
                               snn::kHsSmemBytes, stream, ph);
    if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
    return SNN_OK;
  }
  // General kernel: spikes leave by TMA stores when each half-tile of 32
  // pixels is a box in (w, h, image) -- tiles of 64 pixels made of whole rows
  // or whole images.
  if (spikes && p.tw * p.th * p.tn == snn::kBN) {
    int bw = 0, bh = 0, bn = 0;
    if (p.tw >= 32) { if (p.tw % 32 == 0) { bw = 32; bh = 1; bn = 1; } }
    else if (p.tw * p.th >= 32) { if (32 % p.tw == 0) { bw = p.tw; bh = 32 / p.tw; bn = 1; } }
    else if (32 % (p.tw * p.th) == 0) { bw = p.tw; bh = p.th; bn = 32 / (p.tw * p.th); }
    if (bw > 0) {
      const size_t F = d->Cout, OW = g.OW, OH = g.OH, B = d->B;
      cuuint64_t odims[5] = {F, OW, OH, B, static_cast<cuuint64_t>(d->T)};
      cuuint64_t ostrides[4] = {F * 2, OW * F * 2, OH * OW * F * 2, B * OH * OW * F * 2};
      cuuint32_t obox[5] = {32, static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh),
                            static_cast<cuuint32_t>(bn), 1};
      if ((st = encode(&p.tmap_out, 5, out, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
      p.tma_out = 1;
    }
  }
  if (pair) {
    const int n_pairs = p.n_m / 2;
    const int per_pair = std::max(1, std::min(p.n_px_tiles, (g_num_sms / 2) / n_pairs));
    const long long grid = 2LL * per_pair * n_pairs;
    if (grid > 0x7fffffffLL) return fail(SNN_E_INVALID, "grid too large");
    cudaError_t e = launch_pdl_pair(conv_pair_kernel_fn(mode, rm), dim3(static_cast<unsigned>(grid)),
                                    dim3(snn::kThreads), snn::GenCfg<4, true>::kSmemBytes, stream, p);
    if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
    return SNN_OK;
  }
  const int per_m = std::max(1, std::min(p.n_px_tiles, g_num_sms / p.n_m));
  const long long grid = static_cast<long long>(per_m) * p.n_m;
  if (grid > 0x7fffffffLL) return fail(SNN_E_INVALID, "grid too large");
  cudaError_t e = launch_pdl(conv_kernel_fn(mode, rm, tc, g.kdup > 1),
                             dim3(static_cast<unsigned>(grid)), dim3(snn::kThreads),
                             conv_smem_bytes(tc, g.kdup > 1), stream, p);
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
  return SNN_OK;
}

}  // namespace

namespace {
using GlueKernel = void (*)(const snn::GlueParams);
template <bool POOL, int KS = 0, typename I = long long>
GlueKernel glue_fn(int mode) {
  if (mode == snn::kModeLifHalf) return snn::glue_neuron_kernel<snn::kModeLifHalf, POOL, KS, I>;
  if (mode == snn::kModeLifDiv) return snn::glue_neuron_kernel<snn::kModeLifDiv, POOL, KS, I>;
  if constexpr (POOL)
    if (mode == snn::kModeNone) return snn::glue_neuron_kernel<snn::kModeNone, true, KS, I>;
  return snn::glue_neuron_kernel<snn::kModeIf, POOL, KS, I>;
}
// 32-bit element indices where the grid-stride loop stays below 2^31.
template <bool POOL, int KS = 0>
GlueKernel glue_fn_sized(int mode, bool small) {
  return small ? glue_fn<POOL, KS, int>(mode) : glue_fn<POOL, KS, long long>(mode);
}

// Shared checks and launch of the Add / MaxPool + neuron glue; one_input:
// the neuron of `a` alone (b unused).
int launch_glue(const snn_conv_desc* d, bool pool, const void* a, const void* b, float* state,
                void* out, void* stream, bool one_input = false) {
  int st = ensure_init();
  if (st) return st;
  if (!d || !a || (!pool && !one_input && !b) || !out) return fail(SNN_E_INVALID, "null pointer");
  if (one_input) b = nullptr;
  if (d->T < 1 || d->B < 1 || d->H < 1 || d->W < 1 || d->Cout < 8 || d->Cout % 8)
    return fail(SNN_E_INVALID, "bad shape (channels a positive multiple of 8)");
  const bool no_neuron = pool && d->neuron == SNN_NEURON_NONE;   // plain max pool
  if (d->neuron != SNN_NEURON_LIF && d->neuron != SNN_NEURON_IF && !no_neuron)
    return fail(SNN_E_INVALID, pool ? "neuron must be LIF, IF or NONE" : "neuron must be LIF or IF");
  if (d->neuron == SNN_NEURON_LIF && !(d->tau > 0.0f)) return fail(SNN_E_INVALID, "tau must be positive");
  if ((d->flags & (SNN_FLAG_READ_STATE | SNN_FLAG_WRITE_STATE)) && !state)
    return fail(SNN_E_INVALID, "state flags set but state is null");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(SNN_E_INVALID, "tensors must be 16-byte aligned");
  const bool bits = (d->flags & SNN_FLAG_SPIKE_BITS) != 0;
  if (bits && (!pool || !no_neuron || d->Cout % 16 ||
               (d->flags & (SNN_FLAG_READ_STATE | SNN_FLAG_WRITE_STATE))))
    return fail(SNN_E_INVALID, "bit-packed input: plain max pool (SNN_NEURON_NONE, no state) of "
                               "a multiple of 16 channels only");
  snn::GlueParams p;
  memset(&p, 0, sizeof(p));
  p.a = static_cast<const __half*>(a);
  p.b = static_cast<const __half*>(b);
  p.out = static_cast<__half*>(out);
  p.state = state;
  p.T = d->T; p.B = d->B; p.H = d->H; p.W = d->W; p.C = d->Cout; p.flags = d->flags;
  if (pool) {
    if (d->Cin != d->Cout) return fail(SNN_E_INVALID, "max pool keeps the channel count (Cin == Cout)");
    if (d->KH < 1 || d->KW < 1 || d->stride < 1 || d->pad < 0 || 2 * d->pad > std::min(d->KH, d->KW))
      return fail(SNN_E_INVALID, "bad pool window (pad at most half the window)");
    p.KH = d->KH; p.KW = d->KW; p.stride = d->stride; p.pad = d->pad;
    p.OH = (d->H + 2 * d->pad - d->KH) / d->stride + 1;
    p.OW = (d->W + 2 * d->pad - d->KW) / d->stride + 1;
    if (p.OH < 1 || p.OW < 1) return fail(SNN_E_INVALID, "empty output");
  } else {
    p.OH = d->H; p.OW = d->W;
  }
  const long long total_in = static_cast<long long>(d->T) * d->B * d->H * d->W * d->Cout;
  if (total_in > (1LL << 40)) return fail(SNN_E_INVALID, "tensors too large");
  p.tau = d->tau;
  // Reference computes (1.0 - 1.0/tau) in double, then float32 (models/neurons.py:125).
  p.decay = d->neuron == SNN_NEURON_LIF ? static_cast<float>(1.0 - 1.0 / static_cast<double>(d->tau)) : 1.0f;
  p.v_th = d->v_threshold; p.v_reset = d->v_reset;
  const int mode = no_neuron ? snn::kModeNone
                   : d->neuron == SNN_NEURON_IF ? snn::kModeIf
                   : d->tau == 2.0f ? snn::kModeLifHalf : snn::kModeLifDiv;
  if (no_neuron && !bits && static_cast<long long>(d->T) * d->B <= 0x7fffffffLL &&
      static_cast<long long>(d->B) * p.OH * p.OW * (d->Cout / 8) < static_cast<long long>(g_num_sms) * 2048) {
    // The plain pool carries nothing across timesteps: where one thread per
    // (pixel, 8 channels) would not fill the GPU, its T*B images run as
    // independent ones, T times the threads (larger pools keep the timestep
    // loop, which amortises a thread's index arithmetic).
    p.B = d->T * d->B;
    p.T = 1;
  }
  const long long n = static_cast<long long>(p.B) * p.OH * p.OW * (d->Cout / 8);
  const long long blocks = std::max<long long>(1, std::min<long long>((n + 255) / 256,
                                                                    static_cast<long long>(g_num_sms) * 16));
  const bool small = n + blocks * 256 < (1LL << 31);
  GlueKernel k = glue_fn_sized<false>(mode, small);
  if (bits) {
    // Thread = one output pixel of one image (grid y: the T*B images),
    // 32-bit within an image.
    if (static_cast<long long>(d->H) * d->W * (d->Cout / 16) >= (1LL << 30))
      return fail(SNN_E_INVALID, "bit-packed pool: image too large");
    const long long per_img = static_cast<long long>(p.OH) * p.OW;
    const unsigned gxb = static_cast<unsigned>(std::min<long long>((per_img + 255) / 256, 1024));
    const unsigned gyb = static_cast<unsigned>(std::min<long long>(static_cast<long long>(d->T) * d->B, 65535));
    k = (d->KH == 3 && d->KW == 3) ? snn::maxpool_bits_kernel<3>
      : (d->KH == 2 && d->KW == 2) ? snn::maxpool_bits_kernel<2> : snn::maxpool_bits_kernel<0>;
    cudaError_t e = launch_pdl(k, dim3(gxb, gyb), dim3(256), 0, stream, p);
    if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
    return SNN_OK;
  }
  if (pool) {
    // Square 2x2 / 3x3 windows issue all their loads at once.
    k = (d->KH == 3 && d->KW == 3) ? glue_fn_sized<true, 3>(mode, small)
      : (d->KH == 2 && d->KW == 2) ? glue_fn_sized<true, 2>(mode, small) : glue_fn_sized<true>(mode, small);
  }
  cudaError_t e = launch_pdl(k, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, p);
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
  return SNN_OK;
}
}  // namespace

extern "C" {

int snn_abi_version(void) { return SNN_ABI_VERSION; }

int snn_init(void) { return ensure_init(); }

const char* snn_last_error_message(void) { return g_msg; }

int snn_conv_variant(const snn_conv_desc* d) {
  Geometry g;
  int st = check_desc(d, &g);
  if (st) return st;
  return select_variant(d, g);
}

int snn_conv_out_shape(const snn_conv_desc* d, int32_t* OH, int32_t* OW) {
  Geometry g;
  int st = check_desc(d, &g);
  if (st) return st;
  if (OH) *OH = g.OH;
  if (OW) *OW = g.OW;
  return SNN_OK;
}

int snn_conv_weight_bytes(const snn_conv_desc* d, size_t* bytes) {
  Geometry g;
  int st = check_desc(d, &g);
  if (st) return st;
  if (!bytes) return fail(SNN_E_INVALID, "null output");
  *bytes = meta_offset(g) + static_cast<size_t>(g.Fpad / snn::kBM) * (g.Kw / 32) * snn::kBM * 4;
  return SNN_OK;
}

int snn_pack_weight_24(const snn_conv_desc* d, const float* w, void* blob) {
  Geometry g;
  int st = check_desc(d, &g);
  if (st) return st;
  if (!w || !blob) return fail(SNN_E_INVALID, "null pointer");
  const int F = d->Cout, C = d->Cin, KH = d->KH, KW = d->KW, K = g.Kw;
  uint8_t* out = static_cast<uint8_t*>(blob);
  size_t total = 0;
  snn_conv_weight_bytes(d, &total);
  memset(out, 0, total);
  __half* vals = reinterpret_cast<__half*>(out);
  uint32_t* meta = reinterpret_cast<uint32_t*>(out + meta_offset(g));
  // Nibble (i0 | i1<<2) per (row, group); padding rows keep (0,1).
  const int G = K / 4;
  uint8_t* nib = new uint8_t[static_cast<size_t>(g.Fpad) * G];
  memset(nib, 0x4, static_cast<size_t>(g.Fpad) * G);
  if (g.kdup > 1) {
    // Dense weights as two 2:4 halves per activation k-block kb: weight
    // k-block 2kb keeps positions (0,1) of every group of four input
    // channels, 2kb+1 keeps (2,3); both meet the same activations.
    // Channels past Cin (the last k-block's padding) are zero weights with
    // the same fixed pairs.
    for (int f = 0; f < F; ++f)
      for (int kh = 0; kh < KH; ++kh)
        for (int kw = 0; kw < KW; ++kw)
          for (int c0 = 0; c0 < g.cin_blocks * snn::kKB; c0 += 4) {
            const int kb = (kh * KW + kw) * g.cin_blocks + c0 / snn::kKB;
            const int gi = (c0 % snn::kKB) / 4;
            for (int h = 0; h < 2; ++h) {
              const int grp = (kb * 2 + h) * (snn::kKB / 4) + gi;
              for (int u = 0; u < 2; ++u) {
                const int c = c0 + 2 * h + u;
                vals[static_cast<size_t>(f) * (K / 2) + 2 * grp + u] = __float2half_rn(
                    c < C ? w[((static_cast<size_t>(f) * C + c) * KH + kh) * KW + kw] : 0.0f);
              }
              nib[static_cast<size_t>(f) * G + grp] = h ? (2 | (3 << 2)) : (0 | (1 << 2));
            }
          }
  }
  for (int f = 0; f < F && g.kdup == 1; ++f) {
    for (int kh = 0; kh < KH; ++kh) {
      for (int kw = 0; kw < KW; ++kw) {
        for (int c0 = 0; c0 < C; c0 += 4) {
          float v4[4];
          int nz[4], cnt = 0;
          for (int i = 0; i < 4; ++i) {
            v4[i] = w[((static_cast<size_t>(f) * C + c0 + i) * KH + kh) * KW + kw];
            if (v4[i] != 0.f) nz[cnt++] = i;
          }
          if (cnt > 2) {
            delete[] nib;
            return fail(SNN_E_NOT_24, "row %d tap (%d,%d) channels %d..%d: %d non-zeros",
                        f, kh, kw, c0, c0 + 3, cnt);
          }
          // Fill with the lowest unused positions.
          for (int i = 0; cnt < 2 && i < 4; ++i) {
            bool used = false;
            for (int j = 0; j < cnt; ++j) used |= (nz[j] == i);
            if (!used) nz[cnt++] = i;
          }
          if (nz[0] > nz[1]) { int t = nz[0]; nz[0] = nz[1]; nz[1] = t; }
          const int k = (kh * KW + kw) * g.cin_blocks * snn::kKB + c0;   // padded GEMM K index
          const int grp = k / 4;
          vals[static_cast<size_t>(f) * (K / 2) + 2 * grp] = __float2half_rn(v4[nz[0]]);
          vals[static_cast<size_t>(f) * (K / 2) + 2 * grp + 1] = __float2half_rn(v4[nz[1]]);
          nib[static_cast<size_t>(f) * G + grp] = static_cast<uint8_t>(nz[0] | (nz[1] << 2));
        }
      }
    }
  }
  const int J = K / 32;
  for (int mt = 0; mt < g.Fpad / snn::kBM; ++mt) {
    for (int j = 0; j < J; ++j) {
      for (int L = 0; L < snn::kBM; ++L) {
        const int r0 = mt * snn::kBM + 16 * (L / 16) + L % 8;
        const int g0 = (32 * j + 16 * ((L / 8) % 2)) / 4;
        uint32_t word = 0;
        for (int q = 0; q < 4; ++q) {
          word |= static_cast<uint32_t>(nib[static_cast<size_t>(r0) * G + g0 + q]) << (4 * q);
          word |= static_cast<uint32_t>(nib[static_cast<size_t>(r0 + 8) * G + g0 + q]) << (16 + 4 * q);
        }
        meta[(static_cast<size_t>(mt) * J + j) * snn::kBM + L] = word;
      }
    }
  }
  delete[] nib;
  return SNN_OK;
}

int snn_conv_forward(const snn_conv_desc* d, const void* data, const void* weight, float* state,
                     const float* bn_scale, const float* bn_bias, void* out, void* stream) {
  return launch_conv(d, data, weight, state, nullptr, bn_scale, bn_bias, nullptr, snn::kResNone,
                     out, stream);
}

int snn_conv_forward_res(const snn_conv_desc* d, const void* data, const void* weight,
                         float* state, const float* bn_scale, const float* bn_bias,
                         const void* residual, void* out, void* stream) {
  if (!d) return fail(SNN_E_INVALID, "null descriptor");
  if (!residual) return fail(SNN_E_INVALID, "null residual");
  if (d->res_mode != SNN_RES_ADD_AFTER && d->res_mode != SNN_RES_ADD_BEFORE)
    return fail(SNN_E_INVALID, "snn_conv_forward_res takes res_mode ADD_AFTER or ADD_BEFORE");
  return launch_conv(d, data, weight, state, nullptr, bn_scale, bn_bias, residual,
                     d->res_mode == SNN_RES_ADD_BEFORE ? snn::kResAddBefore : snn::kResAddAfter,
                     out, stream);
}

int snn_conv_forward_res2(const snn_conv_desc* d, const void* data, const void* weight,
                          float* state, float* state2, const float* bn_scale,
                          const float* bn_bias, const void* residual, void* out,
                          void* stream) {
  if (!d) return fail(SNN_E_INVALID, "null descriptor");
  if (!residual) return fail(SNN_E_INVALID, "null residual");
  if (d->res_mode != SNN_RES_TWO_NEURON)
    return fail(SNN_E_INVALID, "snn_conv_forward_res2 takes res_mode TWO_NEURON");
  return launch_conv(d, data, weight, state, state2, bn_scale, bn_bias, residual,
                     snn::kResTwoNeuron, out, stream);
}

int snn_conv_tsplit_workspace_bytes(const snn_conv_desc* d, size_t* bytes) {
  Geometry g;
  int st = check_desc(d, &g);
  if (st) return st;
  if (!bytes) return fail(SNN_E_INVALID, "null output");
  *bytes = static_cast<size_t>(d->T) * d->B * g.OH * g.OW * d->Cout * sizeof(float);
  return SNN_OK;
}

int snn_conv_forward_tsplit(const snn_conv_desc* d, const void* data, const void* weight,
                            float* state, const float* bn_scale, const float* bn_bias,
                            const void* residual, void* out, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int st = ensure_init();
  if (st) return st;
  Geometry g;
  if ((st = check_desc(d, &g))) return st;
  if (d->neuron != SNN_NEURON_LIF && d->neuron != SNN_NEURON_IF)
    return fail(SNN_E_INVALID, "timestep split: neuron must be LIF or IF");
  if (d->flags & (SNN_FLAG_DENSE | SNN_FLAG_CTA_PAIR))
    return fail(SNN_E_INVALID, "timestep split: no dense weights or CTA pairs");
  if (residual && d->res_mode != SNN_RES_ADD_AFTER && d->res_mode != SNN_RES_ADD_BEFORE)
    return fail(SNN_E_INVALID, "timestep split: residual ADD_AFTER or ADD_BEFORE");
  if (!out || !workspace) return fail(SNN_E_INVALID, "null tensor pointer");
  if ((d->flags & (SNN_FLAG_READ_STATE | SNN_FLAG_WRITE_STATE)) && !state)
    return fail(SNN_E_INVALID, "state flags set but state is null");
  size_t need = 0;
  snn_conv_tsplit_workspace_bytes(d, &need);
  if (workspace_bytes < need)
    return fail(SNN_E_INVALID, "workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if ((reinterpret_cast<uintptr_t>(workspace) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(residual)) & 15)
    return fail(SNN_E_INVALID, "workspace, out and residual must be 16-byte aligned");
  // Phase 1: conv + BN of all T*B images, no neuron, fp32 into the
  // workspace.  The images are independent here, only the order of the flat
  // [T*B] index matters, so it is regrouped as [T'][B'] to suit the kernel:
  // T' = 1 where the halo kernels then serve it -- the resident-weight halo
  // kernel (timesteps outer, so B' = T*B images give it many tiles), or the
  // streaming halo kernel on 4x4 images (a tile is four whole images) --
  // else T' = 2: two-timestep tiles, twice the CTAs of four-timestep ones.
  // Measured at the DVS shapes (64 images): stage-2 3x3 21.3 (T' = 4) ->
  // 10.3 us, stage-3 19.8 -> 13.8, stage-4 28.6 -> 18.0, strided 3x3
  // 16.4 -> 12.0 and 21.2 -> 16.0 us.
  snn_conv_desc d1 = *d;
  const long long tb = static_cast<long long>(d->T) * d->B;
  d1.neuron = SNN_NEURON_NONE;
  d1.flags = d->flags & SNN_FLAG_FORCE_GENERIC;
  d1.res_mode = SNN_RES_ADD_AFTER;
  d1.T = 1;
  d1.B = static_cast<int32_t>(tb);
  const int v1 = select_variant(&d1, g);
  const bool t1 = v1 == SNN_VARIANT_HALO_RESIDENT ||
                  (v1 == SNN_VARIANT_HALO_STREAM && g.OH == 4 && g.OW == 4);
  d1.T = (t1 || tb % 2) ? 1 : 2;
  d1.B = static_cast<int32_t>(tb / d1.T);
  if ((st = launch_conv(&d1, data, weight, nullptr, nullptr, bn_scale, bn_bias, nullptr,
                        snn::kResNone, workspace, stream)))
    return st;
  // Phase 2: the neuron over T (+ residual), spikes out.
  snn::TsplitParams p;
  memset(&p, 0, sizeof(p));
  p.z = static_cast<const float*>(workspace);
  p.residual = static_cast<const __half*>(residual);
  p.out = static_cast<__half*>(out);
  p.state = state;
  p.P = static_cast<long long>(d->B) * g.OH * g.OW;
  p.T = d->T; p.C = d->Cout; p.flags = d->flags;
  p.tau = d->tau;
  // Reference computes (1.0 - 1.0/tau) in double, then float32 (models/neurons.py:125).
  p.decay = d->neuron == SNN_NEURON_LIF ? static_cast<float>(1.0 - 1.0 / static_cast<double>(d->tau)) : 1.0f;
  p.v_th = d->v_threshold; p.v_reset = d->v_reset;
  const int mode = d->neuron == SNN_NEURON_IF ? snn::kModeIf
                   : d->tau == 2.0f ? snn::kModeLifHalf : snn::kModeLifDiv;
  const int rm = !residual ? snn::kResNone
                 : d->res_mode == SNN_RES_ADD_BEFORE ? snn::kResAddBefore : snn::kResAddAfter;
  using TsK = void (*)(const snn::TsplitParams);
  TsK k = nullptr;
  switch (mode * 3 + (rm == snn::kResNone ? 0 : rm == snn::kResAddAfter ? 1 : 2)) {
    case 0: k = snn::tsplit_neuron_kernel<snn::kModeLifHalf, snn::kResNone>; break;
    case 1: k = snn::tsplit_neuron_kernel<snn::kModeLifHalf, snn::kResAddAfter>; break;
    case 2: k = snn::tsplit_neuron_kernel<snn::kModeLifHalf, snn::kResAddBefore>; break;
    case 3: k = snn::tsplit_neuron_kernel<snn::kModeLifDiv, snn::kResNone>; break;
    case 4: k = snn::tsplit_neuron_kernel<snn::kModeLifDiv, snn::kResAddAfter>; break;
    case 5: k = snn::tsplit_neuron_kernel<snn::kModeLifDiv, snn::kResAddBefore>; break;
    case 6: k = snn::tsplit_neuron_kernel<snn::kModeIf, snn::kResNone>; break;
    case 7: k = snn::tsplit_neuron_kernel<snn::kModeIf, snn::kResAddAfter>; break;
    default: k = snn::tsplit_neuron_kernel<snn::kModeIf, snn::kResAddBefore>; break;
  }
  const long long n = p.P * d->Cout;
  const long long blocks = std::max<long long>(1, std::min<long long>((n + 255) / 256,
                                                                    static_cast<long long>(g_num_sms) * 8));
  cudaError_t e = launch_pdl(k, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, p);
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
  return SNN_OK;
}

// out2 non-null: the dual form (fp16 BN output in `out`, spikes of d->neuron
// on it in `out2`), general tensor-core stem only.
static int stem_forward_impl(const snn_conv_desc* d, int32_t Tin, const float* x, const float* w,
                             const float* bn_scale, const float* bn_bias, void* out, void* out2,
                             void* stream) {
  int st = ensure_init();
  if (st) return st;
  if (!d || !x || !w || !bn_scale || !bn_bias || !out) return fail(SNN_E_INVALID, "null pointer");
  if (d->T < 1 || d->B < 1 || d->Cin < 1 || d->Cout < 16 || d->Cout % 16 || d->Cout > 4096 ||
      d->KH < 1 || d->KW < 1 || d->stride < 1 || d->pad < 0 ||
      static_cast<long long>(d->KH) * d->KW * d->Cin * d->Cout > 12288)
    return fail(SNN_E_INVALID, "unsupported stem geometry (Cout multiple of 16, K*Cout <= 12288)");
  if (Tin != 1 && Tin != d->T) return fail(SNN_E_INVALID, "Tin must be 1 or T");
  if (d->neuron < SNN_NEURON_LIF || d->neuron > SNN_NEURON_NONE)
    return fail(SNN_E_INVALID, "stem neuron must be LIF, IF or NONE (fp16 BN output)");
  if (out2 && d->neuron == SNN_NEURON_NONE)
    return fail(SNN_E_INVALID, "dual stem: the neuron of the spike output must be LIF or IF");
  if (out2 && ((reinterpret_cast<uintptr_t>(out2) & 15) || out2 == out))
    return fail(SNN_E_INVALID, "dual stem: out_spikes must be a separate 16-byte aligned tensor");
  const bool bits = (d->flags & SNN_FLAG_SPIKE_BITS) != 0;
  if (bits && (out2 || d->neuron == SNN_NEURON_NONE))
    return fail(SNN_E_INVALID, "bit-packed stem output: spikes of a LIF or IF neuron, single output");
  const int OH = (d->H + 2 * d->pad - d->KH) / d->stride + 1;
  const int OW = (d->W + 2 * d->pad - d->KW) / d->stride + 1;
  if (OH < 1 || OW < 1) return fail(SNN_E_INVALID, "empty output");
  snn::StemParams p;
  memset(&p, 0, sizeof(p));
  p.x = x; p.w = w; p.scale = bn_scale; p.bias = bn_bias;
  p.out = static_cast<__half*>(out);
  p.T = d->T; p.Tin = Tin; p.B = d->B; p.Cin = d->Cin; p.H = d->H; p.W = d->W;
  p.Cout = d->Cout; p.KH = d->KH; p.KW = d->KW; p.stride = d->stride; p.pad = d->pad;
  p.OH = OH; p.OW = OW; p.neuron = d->neuron;
  p.tau = d->tau; p.decay = static_cast<float>(1.0 - 1.0 / static_cast<double>(d->tau));
  p.v_th = d->v_threshold; p.v_reset = d->v_reset;
  p.err = nullptr;
  p.timeout = 4000000000ull;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p.err), g_device_err) != cudaSuccess)
    return fail(SNN_E_CUDA, "error word address");
  // Tensor-core fast path: 3x3 s1 p1, 64 channels, input repeated over T,
  // rows of at most 128 pixels.
  if (!out2 && !bits && Tin == 1 && d->neuron != SNN_NEURON_NONE && d->KH == 3 && d->KW == 3 && d->stride == 1 &&
      d->pad == 1 && d->Cout == 64 &&
      (d->Cin == 1 || d->Cin == 3) && OW <= snn::kStemPx) {
    const int mode = d->neuron == SNN_NEURON_IF ? snn::kModeIf
                     : d->tau == 2.0f ? snn::kModeLifHalf : snn::kModeLifDiv;
    const int R = snn::kStemPx / OW;
    const size_t smem = static_cast<size_t>(snn::stem_tc_smem_bytes(d->Cin, R, OW));
    // Persistent blocks (three per SM: registers), each walking row tiles.
    const long long n_tiles = static_cast<long long>(d->B) * ((OH + R - 1) / R);
    const long long nblk = std::min<long long>(n_tiles, 3LL * g_num_sms);
    if (smem <= static_cast<size_t>(kStemTcSmemMax) && n_tiles <= 0x7fffffffLL) {
      // Spike tiles leave by TMA stores: (64 ch, OW, OH, B, T), box {64, OW, R, 1, 1}.
      const cuuint64_t odims[5] = {64, static_cast<cuuint64_t>(OW), static_cast<cuuint64_t>(OH),
                                   static_cast<cuuint64_t>(d->B), static_cast<cuuint64_t>(d->T)};
      const cuuint64_t ostrides[4] = {64 * 2, static_cast<cuuint64_t>(OW) * 64 * 2,
                                      static_cast<cuuint64_t>(OH) * OW * 64 * 2,
                                      static_cast<cuuint64_t>(d->B) * OH * OW * 64 * 2};
      const cuuint32_t obox[5] = {64, static_cast<cuuint32_t>(OW), static_cast<cuuint32_t>(R), 1, 1};
      if ((reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
          encode(&p.tmap_out, 5, out, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_128B) == SNN_OK)
        p.tma_out = 1;
      cudaError_t e = launch_pdl(stem_tc_fn(d->Cin, mode), dim3(static_cast<unsigned>(nblk)),
                                 dim3(snn::kStemThreads), smem, stream, p);
      if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
      return SNN_OK;
    }
  }
  // General tensor-core stem: any window and stride, per-timestep or
  // repeated input, up to 64 channels and K = Cin*KH*KW <= 192 (warp-specialised, one block per SM).
  const int Kst = d->Cin * d->KH * d->KW;
  const int TWst = std::min(OW, 128), Rst = 128 / TWst;
  const int IRst = (Rst - 1) * d->stride + d->KH, ICst = (TWst - 1) * d->stride + d->KW;
  // Input windows by TMA where the fp32 rows allow it (16-byte row pitch, W % 4
  // == 0): the box starts at the window's first column rounded down to 16
  // bytes, so it is up to 3 columns wider, rounded up to 16 bytes.
  const int ICp = (ICst + 6) & ~3;
  const bool tma_in = d->W % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ICp <= 256 &&
                      IRst <= 256 && d->Cin <= 256 &&
                      4LL * d->Cin * IRst * ICp <= snn::kStemGMaxStage;
  const long long stage_bytes = 4LL * d->Cin * IRst * (tma_in ? ICp : ICst);
  const long long units = static_cast<long long>(d->B) * ((OH + Rst - 1) / Rst) *
                          ((OW + TWst - 1) / TWst) * (Tin > 1 ? d->T : 1);
  if (d->Cout <= 64 && Kst <= snn::kStemGMaxK && stage_bytes <= snn::kStemGMaxStage &&
      units < 0x7fffffffLL) {
    p.in_pitch = tma_in ? ICp : ICst;
    if (tma_in) {
      const cuuint64_t idims[5] = {static_cast<cuuint64_t>(d->W), static_cast<cuuint64_t>(d->H),
                                   static_cast<cuuint64_t>(d->Cin), static_cast<cuuint64_t>(d->B),
                                   static_cast<cuuint64_t>(Tin)};
      const cuuint64_t row = static_cast<cuuint64_t>(d->W) * 4;
      const cuuint64_t istrides[4] = {row, row * d->H, row * d->H * d->Cin,
                                      row * d->H * d->Cin * d->B};
      const cuuint32_t ibox[5] = {static_cast<cuuint32_t>(ICp), static_cast<cuuint32_t>(IRst),
                                  static_cast<cuuint32_t>(d->Cin), 1, 1};
      if ((st = encode(&p.tmap_in, 5, x, idims, istrides, ibox, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
        return st;
      p.tma_in = 1;
    }
    const int mode = d->neuron == SNN_NEURON_NONE ? snn::kModeNone
                     : d->neuron == SNN_NEURON_IF ? snn::kModeIf
                     : d->tau == 2.0f ? snn::kModeLifHalf : snn::kModeLifDiv;
    const int nk = (Kst + 31) / 32;
    const size_t smem = static_cast<size_t>(snn::stem_tcg_smem_bytes(nk));
    const long long n_tiles = static_cast<long long>(d->B) * ((OH + Rst - 1) / Rst) *
                              ((OW + TWst - 1) / TWst);
    const long long nblk = std::max<long long>(1, std::min<long long>(n_tiles, g_num_sms));
    if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      p.out2 = static_cast<__half*>(out2);
      p.bits_out = bits ? 1 : 0;
      cudaError_t e = launch_pdl(stem_tcg_fn(mode, out2 != nullptr), dim3(static_cast<unsigned>(nblk)),
                                 dim3(snn::kStemGThreads), smem, stream, p);
      if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
      return SNN_OK;
    }
  }
  if (out2 || bits)
    return fail(SNN_E_INVALID, "dual or bit-packed stem needs the general tensor-core stem (Cout <= 64, "
                "Cin*KH*KW <= %d, staged window <= %d bytes, out 16-byte aligned)",
                snn::kStemGMaxK, snn::kStemGMaxStage);
  const long long pixels = static_cast<long long>(d->B) * OH * OW;
  const int px_per_block = 256 / (d->Cout / 16);
  if (px_per_block < 1) return fail(SNN_E_INVALID, "stem Cout too large");
  const long long nblk = std::min<long long>((pixels + px_per_block - 1) / px_per_block,
                                             static_cast<long long>(g_num_sms) * 2);
  dim3 block(256);
  dim3 grid(static_cast<unsigned>(nblk));
  const size_t smem = static_cast<size_t>(d->KH) * d->KW * d->Cin * d->Cout * sizeof(float);
  StemKernel k = (d->KH == 3 && d->KW == 3 && d->Cin == 3)   ? snn::stem_conv_lif_kernel<3, 3>
                 : (d->KH == 3 && d->KW == 3 && d->Cin == 2) ? snn::stem_conv_lif_kernel<3, 2>
                                                             : snn::stem_conv_lif_kernel<0, 0>;
  cudaError_t e = launch_pdl(k, grid, block, smem, stream, p);
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
  return SNN_OK;
}

int snn_stem_forward(const snn_conv_desc* d, int32_t Tin, const float* x, const float* w,
                     const float* bn_scale, const float* bn_bias, void* out, void* stream) {
  return stem_forward_impl(d, Tin, x, w, bn_scale, bn_bias, out, nullptr, stream);
}

int snn_stem_forward_dual(const snn_conv_desc* d, int32_t Tin, const float* x, const float* w,
                          const float* bn_scale, const float* bn_bias, void* out_bn,
                          void* out_spikes, void* stream) {
  if (!out_spikes) return fail(SNN_E_INVALID, "null pointer");
  return stem_forward_impl(d, Tin, x, w, bn_scale, bn_bias, out_bn, out_spikes, stream);
}

int snn_head_forward(int32_t T, int32_t B, int32_t HW, int32_t C, int32_t NC, const void* x,
                     const float* fc_w, const float* fc_b, float* logits, void* stream) {
  int st = ensure_init();
  if (st) return st;
  if (!x || !fc_w || !logits) return fail(SNN_E_INVALID, "null pointer");
  if (T < 1 || B < 1 || HW < 1 || C < 8 || C % 8 || C > 704 || NC < 1)
    return fail(SNN_E_INVALID, "bad head shape (C multiple of 8, <= 704)");
  if (reinterpret_cast<uintptr_t>(x) & 15) return fail(SNN_E_INVALID, "x must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(fc_w) & 15) return fail(SNN_E_INVALID, "fc_w must be 16-byte aligned");
  const int threads = 1024;
  const size_t smem = static_cast<size_t>(snn::kHeadSlots + 1) * C * sizeof(float);
  cudaError_t e = launch_pdl(snn::head_pool_fc_kernel, dim3(B), dim3(threads), smem, stream,
                             static_cast<const __half*>(x), fc_w, fc_b, logits, T, B, HW, C, NC);
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
  return SNN_OK;
}

int snn_add_lif_forward(const snn_conv_desc* d, const void* a, const void* b, float* state,
                        void* out, void* stream) {
  return launch_glue(d, false, a, b, state, out, stream);
}

int snn_maxpool_lif_forward(const snn_conv_desc* d, const void* x, float* state, void* out,
                            void* stream) {
  return launch_glue(d, true, x, nullptr, state, out, stream);
}

int snn_lif_forward(const snn_conv_desc* d, const void* x, float* state, void* out, void* stream) {
  return launch_glue(d, false, x, nullptr, state, out, stream, true);
}

int snn_spikformer_attn_forward(int32_t T, int32_t B, int32_t N, int32_t heads,
                                int32_t head_dim, float scale, float tau, float v_threshold,
                                float v_reset, int32_t flags, const void* q, const void* k,
                                const void* v, float* state, void* out, void* stream) {
  int st = ensure_init();
  if (st) return st;
  if (!q || !k || !v || !out) return fail(SNN_E_INVALID, "null tensor pointer");
  if (T < 1 || B < 1 || heads < 1 || N < 1 || N > snn::kAttnMaxN)
    return fail(SNN_E_INVALID, "bad attention shape (1 <= N <= %d)", snn::kAttnMaxN);
  if (head_dim != 32 && head_dim != 64) return fail(SNN_E_INVALID, "head_dim must be 32 or 64");
  if (!(tau > 0.0f)) return fail(SNN_E_INVALID, "tau must be positive");
  if ((flags & (SNN_FLAG_READ_STATE | SNN_FLAG_WRITE_STATE)) && !state)
    return fail(SNN_E_INVALID, "state flags set but state is null");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(SNN_E_INVALID, "q, k, v and out must be 16-byte aligned");
  const long long TB = static_cast<long long>(T) * B;
  const long long C = static_cast<long long>(heads) * head_dim;
  if (TB * N * C * ((flags & SNN_FLAG_QKV_PACKED) ? 3 : 1) > 0x7fffffffLL ||
      static_cast<long long>(B) * heads > 0x7fffffffLL)
    return fail(SNN_E_INVALID, "attention tensors too large");
  snn::AttnParams p;
  memset(&p, 0, sizeof(p));
  p.kv_rows = (N + 15) / 16 * 16;
  {
    // q, k, v as 3-D {C, N, T*B}; q boxes are 128-token M-tiles, k/v boxes
    // all kv_rows tokens (rows past N read as zero).
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(N),
                          static_cast<cuuint64_t>(TB)};
    // SNN_FLAG_QKV_PACKED: rows of 3C elements (q | k | v of one token).
    const long long ld = (flags & SNN_FLAG_QKV_PACKED) ? 3 * C : C;
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, static_cast<cuuint64_t>(N * ld) * 2};
    const CUtensorMapSwizzle swz =
        head_dim == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    cuuint32_t box_q[3] = {static_cast<cuuint32_t>(head_dim),
                           static_cast<cuuint32_t>(std::min<int>(N, 128)), 1};
    cuuint32_t box_kv[3] = {static_cast<cuuint32_t>(head_dim), static_cast<cuuint32_t>(p.kv_rows), 1};
    if ((st = encode(&p.tmap_q, 3, q, dims, strides, box_q, swz))) return st;
    if ((st = encode(&p.tmap_k, 3, k, dims, strides, box_kv, swz))) return st;
    if ((st = encode(&p.tmap_v, 3, v, dims, strides, box_kv, swz))) return st;
    if (head_dim == 32) {
      // Spikes leave by TMA stores of {32 channels, 32 tokens} tiles: out as
      // 4-D {C, N, B, T} (tokens past N are not written).
      if (reinterpret_cast<uintptr_t>(out) & 15) return fail(SNN_E_INVALID, "out must be 16-byte aligned");
      cuuint64_t odims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(N),
                             static_cast<cuuint64_t>(B), static_cast<cuuint64_t>(T)};
      cuuint64_t ostrides[3] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(N * C) * 2,
                                static_cast<cuuint64_t>(B) * N * C * 2};
      cuuint32_t obox[4] = {32, 32, 1, 1};
      if ((st = encode(&p.tmap_out, 4, out, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
    }
  }
  p.out = static_cast<__half*>(out);
  p.state = state;
  unsigned* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_device_err) != cudaSuccess)
    return fail(SNN_E_CUDA, "error word address");
  p.err = err;
  p.T = T; p.B = B; p.N = N; p.heads = heads; p.C = static_cast<int>(C); p.flags = flags;
  p.scale = scale; p.tau = tau; p.v_th = v_threshold; p.v_reset = v_reset;
  p.lif_half = tau == 2.0f;
  // Reference computes (1.0 - 1.0/tau) in double, then float32 (models/neurons.py:125).
  p.decay = static_cast<float>(1.0 - 1.0 / static_cast<double>(tau));
  p.timeout = 4000000000ull;
  // Persistent: one CTA per SM (about 200 KB of shared memory each) walks
  // the (image, head) items.
  const dim3 grid(static_cast<unsigned>(std::min<long long>(static_cast<long long>(B) * heads,
                                                            g_num_sms)));
  cudaError_t e = head_dim == 32
      ? launch_pdl(snn::spikformer_attn_lif_kernel<32>, grid, dim3(snn::kAttnThreads),
                   snn::AttnCfg<32>::kSmemBytes, stream, p)
      : launch_pdl(snn::spikformer_attn_lif_kernel<64>, grid, dim3(snn::kAttnThreads),
                   snn::AttnCfg<64>::kSmemBytes, stream, p);
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "launch: %s", cudaGetErrorString(e));
  return SNN_OK;
}

int snn_get_device_error(uint32_t* code, int reset) {
  int st = ensure_init();
  if (st) return st;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "synchronize: %s", cudaGetErrorString(e));
  unsigned v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_err, sizeof(v));
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "read error word: %s", cudaGetErrorString(e));
  if (code) *code = v;
  if (reset) {
    unsigned z = 0;
    e = cudaMemcpyToSymbol(g_device_err, &z, sizeof(z));
    if (e != cudaSuccess) return fail(SNN_E_CUDA, "clear error word: %s", cudaGetErrorString(e));
  }
  return SNN_OK;
}

}  // extern "C"

// ------------------------------------------------ timestep split, no allocation
// Some callers of this library cannot call cudaMalloc: a runtime that owns
// every device allocation through its own pool or arena, or a host that loads
// the library into a process where allocating is not allowed once serving
// has started.  For them the timestep-split layer has a form whose fp32
// intermediate lives in a fixed array inside the library, so the caller
// passes only inputs and outputs.
namespace {

// 8 MiB of BN outputs: a DVS SEW-ResNet-18 layer at T = 16 and 4 images per
// GPU needs at most 16*4*16*16*128 fp32 (stage 2).  Every GPU that loads the
// library holds the array until the process exits.
constexpr size_t kTsplitStaticBytes = SNN_TSPLIT_STATIC_MAX_BYTES;
static __device__ __align__(256) float g_tsplit_scratch[kTsplitStaticBytes / sizeof(float)];

// Device address of g_tsplit_scratch per device (the name is only a host
// stand-in for it), resolved once per device with that device current.
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int tsplit_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SNN_E_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(SNN_E_INVALID, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_tsplit_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(SNN_E_CUDA, "scratch array address: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return SNN_OK;
}

}  // namespace

extern "C" int snn_conv_forward_tsplit_static(const snn_conv_desc* d, const void* data,
                                              const void* weight, float* state,
                                              const float* bn_scale, const float* bn_bias,
                                              const void* residual, void* out, void* stream) {
  int st = ensure_init();
  if (st) return st;
  size_t need = 0;
  if ((st = snn_conv_tsplit_workspace_bytes(d, &need))) return st;
  if (need > kTsplitStaticBytes)
    return fail(SNN_E_INVALID,
                "layer needs %zu bytes of intermediate, the static array holds %zu "
                "(snn_conv_forward_tsplit with a caller workspace has no limit)",
                need, kTsplitStaticBytes);
  void* scratch = nullptr;
  if ((st = tsplit_scratch_address(&scratch))) return st;
  // Phase 1 writes every element of the region that phase 2 reads, so the
  // previous call's contents never leak into this one.
  return snn_conv_forward_tsplit(d, data, weight, state, bn_scale, bn_bias, residual, out, scratch,
                                 kTsplitStaticBytes, stream);
}

#include "snn_engine.cuh"
