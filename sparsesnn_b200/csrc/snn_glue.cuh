// Memory-bound glue around the fused sparse layers of an SNN ResNet:
//  * stem_tc_kernel / stem_conv_lif_kernel: dense conv (small Cin, e.g. RGB)
//    + BN + LIF/IF over T, computed once when the input is repeated over T
//    (direct encoding) and written as fp16 NHWC spikes per timestep
//    (tensor-core fast path for 3x3 / 64-channel stems; the general CUDA-core
//    kernel covers other shapes and per-timestep inputs).
//  * head_pool_fc_kernel: global average pool + mean over T + linear head.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include "snn_conv.cuh"

namespace snn {

struct StemParams {
  CUtensorMap tmap_out;  // tensor-core path: spikes (64 ch, OW, OH, B, T), box {64, OW, rows, 1, 1}
  CUtensorMap tmap_in;   // general tensor-core path: x as (W, H, Cin, B, Tin) fp32, box {ICp, IR, Cin, 1, 1}
  const float* x;      // [Tin][B][Cin][H][W] fp32
  const float* w;      // [Cout][Cin][KH][KW] fp32
  const float* scale;  // [Cout]
  const float* bias;   // [Cout]
  __half* out;         // [T][B][OH][OW][Cout]
  int T, Tin, B, Cin, H, W, Cout, KH, KW, stride, pad, OH, OW, neuron;
  float tau, decay, v_th, v_reset;
  unsigned* err;                  // device error word (tensor-core path)
  unsigned long long timeout;     // bounded-wait budget, SM cycles
  int tma_out;                    // tensor-core path: spike tiles leave by TMA stores
  int tma_in;                     // general tensor-core path: input windows arrive by TMA
  int in_pitch;                   // general path: staged row pitch (ICp with TMA, else IC)
  __half* out2;                   // general path, dual output: spikes of the fp16 BN output
  int bits_out;                   // general path: `out` holds bit-packed spikes [T][B][OH][OW][Cout/8]
};

// One thread = one output pixel x 16 consecutive output channels
// (Cout/16 threads per pixel, 256 threads per block).  Weights are staged in
// shared memory as [k][cout] (dynamic smem = K*Cout floats, K = Cin*KH*KW);
// the receptive field is gathered once into registers (KS, CIN compile-time
// in the fast instantiation; KS = CIN = 0 selects runtime sizes), and each
// timestep's 16 spikes leave as two 16-byte stores.
template <int KS, int CIN>
__global__ void __launch_bounds__(256, 2)
stem_conv_lif_kernel(const StemParams p) {
  extern __shared__ float ws[];
  pdl_launch_dependents();
  pdl_wait();
  const int KH = KS ? KS : p.KH, KW = KS ? KS : p.KW, Cin = CIN ? CIN : p.Cin;
  const int K = KH * KW * Cin;
  // Coalesced read of the [Cout][K] source, transposed into [K][Cout].
  for (int i = threadIdx.x; i < K * p.Cout; i += blockDim.x) {
    const int co = i / K, k = i - co * K;
    // k = (ci*KH + kh)*KW + kw, matching the [Cout][Cin][KH][KW] source.
    ws[k * p.Cout + co] = p.w[i];
  }
  __syncthreads();
  const int groups = p.Cout / 16;
  const int px_per_block = blockDim.x / groups;
  const int g = threadIdx.x % groups;
  const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
  if (threadIdx.x >= px_per_block * groups) return;
  // Persistent blocks: the staged weights serve many pixel chunks.
  for (long long pix = static_cast<long long>(blockIdx.x) * px_per_block + threadIdx.x / groups;
       pix < P; pix += static_cast<long long>(gridDim.x) * px_per_block) {
  const int ow = static_cast<int>(pix % p.OW);
  const int oh = static_cast<int>((pix / p.OW) % p.OH);
  const int b = static_cast<int>(pix / (static_cast<long long>(p.OW) * p.OH));
  const int c0 = g * 16;
  float v[16], xb[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) { v[j] = 0.f; xb[j] = 0.f; }
  const int ih0 = oh * p.stride - p.pad, iw0 = ow * p.stride - p.pad;
  for (int t = 0; t < p.T; ++t) {
    if (t == 0 || p.Tin > 1) {
      const float* xin = p.x + (static_cast<size_t>(p.Tin > 1 ? t : 0) * p.B + b) *
                                   static_cast<size_t>(Cin) * p.H * p.W;
      float acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = 0.f;
#pragma unroll
      for (int ci = 0; ci < (CIN ? CIN : 1); ++ci) {
        for (int cr = 0; cr < (CIN ? 1 : Cin); ++cr) {
          const int c = CIN ? ci : cr;
#pragma unroll
          for (int kh = 0; kh < (KS ? KS : 1); ++kh) {
            for (int khr = 0; khr < (KS ? 1 : KH); ++khr) {
              const int kk = KS ? kh : khr;
              const int ih = ih0 + kk;
              const bool hok = ih >= 0 && ih < p.H;
#pragma unroll
              for (int kw = 0; kw < (KS ? KS : 1); ++kw) {
                for (int kwr = 0; kwr < (KS ? 1 : KW); ++kwr) {
                  const int ll = KS ? kw : kwr;
                  const int iw = iw0 + ll;
                  const float xv = (hok && iw >= 0 && iw < p.W)
                                       ? __ldg(xin + (static_cast<size_t>(c) * p.H + ih) * p.W + iw) : 0.f;
                  const float* wr = ws + ((c * KH + kk) * KW + ll) * p.Cout + c0;
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const float4 w4 = *reinterpret_cast<const float4*>(wr + 4 * q);
                    acc[4 * q + 0] = fmaf(xv, w4.x, acc[4 * q + 0]);
                    acc[4 * q + 1] = fmaf(xv, w4.y, acc[4 * q + 1]);
                    acc[4 * q + 2] = fmaf(xv, w4.z, acc[4 * q + 2]);
                    acc[4 * q + 3] = fmaf(xv, w4.w, acc[4 * q + 3]);
                  }
                }
              }
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) xb[j] = fmaf(acc[j], __ldg(p.scale + c0 + j), __ldg(p.bias + c0 + j));
    }
    uint32_t packed[8];
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      uint32_t bits = 0;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (p.neuron == 2) {           // no neuron: the BN output in fp16
          bits |= static_cast<uint32_t>(__half_as_ushort(__float2half_rn(xb[j + u]))) << (16 * u);
          continue;
        }
        float h;
        if (p.neuron == 0) h = __fadd_rn(__fmul_rn(v[j + u], p.decay), __fdiv_rn(xb[j + u], p.tau));
        else h = __fadd_rn(v[j + u], xb[j + u]);
        const bool s = h >= p.v_th;
        v[j + u] = s ? p.v_reset : h;
        bits |= (s ? 0x3C00u : 0u) << (16 * u);
      }
      packed[j / 2] = bits;
    }
    uint4* op = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(t) * P + pix) * p.Cout + c0);
    op[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    op[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  }
  }
}

// Tensor-core stem for the direct-encoding case (input repeated over T) of
// a 3x3 stride-1 pad-1 conv with 64 output channels and Cin <= 3, on images
// at most 128 pixels wide.  A block computes R = 128 / OW whole output rows
// of one image as one M = 128 (pixels) x N = 64 (channels) x K = 32 GEMM:
//  * A = im2col of the zero-padded input rows: row = pixel, column
//    k = (ci*3 + kh)*3 + kw (9*Cin taps, zero beyond), fp32 K-major with
//    128-byte swizzle; B = the weights [64][32], same layout;
//  * 3xTF32: each fp32 operand is split into hi = tf32(x) and lo = x - hi,
//    and D = lo*hi + hi*lo + hi*hi with kind::tf32 MMAs accumulating in fp32
//    TMEM (the dropped lo*lo term and lo's own tf32 rounding are below fp32
//    resolution of the sum), so the result matches an fp32 conv to within
//    accumulation order;
//  * epilogue: thread = pixel (TMEM lane), 64 channels: BN once, then LIF/IF
//    over T in registers; each timestep's spikes go to a [128 px][64 ch]
//    fp16 tile (128-byte rows, 16-byte chunks XOR-ed with px & 7) in the A
//    tiles' space and leave as coalesced 16-byte stores (the block's output
//    rows are contiguous in the NHWC tensor).  Two tiles alternate, so one
//    barrier per timestep suffices.
constexpr int kStemPx = 128;
constexpr int kStemThreads = 128;
constexpr int kStemATile = kStemPx * 128;          // [128 px][32 fp32]
constexpr int kStemBTile = 64 * 128;               // [64 ch][32 fp32]
constexpr int kStemXsOffset = 2 * kStemATile + 2 * kStemBTile;   // input rows (floats) start here

// Dynamic shared memory of stem_tc_kernel (bytes, before 1024 alignment).
__host__ __device__ constexpr int stem_tc_smem_bytes(int cin, int R, int OW) {
  return kStemXsOffset + ((cin * (R + 2) * (OW + 2) + 3) / 4 * 4 + 128) * 4 + 64 + 1024;
}

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// Byte offset of fp32 element k of row r in a K-major tile of 128-byte rows
// with 128-byte swizzle.
__device__ __forceinline__ int sw128_f32(int r, int k) {
  return r * 128 + ((((k >> 2) ^ (r & 7))) << 4) + (k & 3) * 4;
}

template <int CIN, int MODE>
__global__ void __launch_bounds__(kStemThreads, 3)
stem_tc_kernel(const __grid_constant__ StemParams p) {
  static_assert(9 * CIN <= 32, "stem K must fit one 32-wide tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sAh = smem;                                  // later: spike tiles
  uint8_t* sAl = smem + kStemATile;
  uint8_t* sBh = smem + 2 * kStemATile;
  uint8_t* sBl = sBh + kStemBTile;
  const int OW = p.OW, R = kStemPx / OW, OWp = OW + 2;
  const int HWp = (R + 2) * OWp;
  float* xs = reinterpret_cast<float*>(smem + kStemXsOffset);   // [CIN][R+2][OW+2]
  float* sc = xs + (CIN * HWp + 3) / 4 * 4;                     // [64]
  float* bi = sc + 64;                                          // [64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(bi + 64);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int bpi = (p.OH + R - 1) / R;                 // row blocks per image
  const int n_tiles = p.B * bpi;
  const int tid = threadIdx.x, warp = tid / 32;

  if (tid == 0) { mbar_init(bar, 1); fence_mbar_init(); }
  if (warp == 0) { tmem_alloc(tmem_slot, 64); tmem_relinquish(); }
  // Weights (constant data, once per persistent block): B[co][k] = w[co][k]
  // for k < 9*CIN, split hi/lo.
  for (int i = tid; i < 64 * 32; i += kStemThreads) {
    const int co = i >> 5, k = i & 31;
    const float wv = k < 9 * CIN ? __ldg(p.w + co * 9 * CIN + k) : 0.f;
    const float hi = to_tf32(wv);
    *reinterpret_cast<float*>(sBh + sw128_f32(co, k)) = hi;
    *reinterpret_cast<float*>(sBl + sw128_f32(co, k)) = wv - hi;
  }
  if (tid < 64) {
    // BN pre-scaled by 1/2 for the tau = 2 LIF step, as in the conv epilogues.
    sc[tid] = MODE == kModeLifHalf ? p.scale[tid] * 0.5f : p.scale[tid];
    bi[tid] = MODE == kModeLifHalf ? p.bias[tid] * 0.5f : p.bias[tid];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();                                         // input and output belong to the stream

  const int px = tid;
  const int r = px / OW, c = px - (px / OW) * OW;
  const bool in_tile = px < R * OW;
  const long long P = static_cast<long long>(p.B) * p.OH * OW;
  bool ok = true;
  int iter = 0;
  // Persistent: tile = R output rows of one image.
  for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++iter) {
    const int b = tile / bpi, oh0 = (tile % bpi) * R;
    const float* xin = p.x + static_cast<size_t>(b) * CIN * p.H * p.W;
    for (int i = tid; i < CIN * HWp; i += kStemThreads) {
      const int ci = i / HWp, rem = i - ci * HWp;
      const int rr = rem / OWp, cc = rem - rr * OWp;
      const int ih = oh0 - 1 + rr, iw = cc - 1;
      xs[i] = (ih >= 0 && ih < p.H && iw >= 0 && iw < p.W)
                  ? __ldg(xin + (static_cast<size_t>(ci) * p.H + ih) * p.W + iw) : 0.f;
    }
    // The previous tile's spike tiles (the A tiles) must be read out before
    // the im2col rows below overwrite them.
    if (p.tma_out && tid == 0) bulk_wait_group_read<0>();
    __syncthreads();                                  // xs ready; the previous tile's spike tiles are out
    // im2col row of this thread's pixel, split hi/lo.
#pragma unroll
    for (int k4 = 0; k4 < 8; ++k4) {
      float hi[4], lo[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = 4 * k4 + j;
        float xv = 0.f;
        if (k < 9 * CIN && in_tile) {
          const int ci = k / 9, kh = (k % 9) / 3, kw = k % 3;
          xv = xs[ci * HWp + (r + kh) * OWp + c + kw];
        }
        hi[j] = to_tf32(xv);
        lo[j] = xv - hi[j];
      }
      const int off = px * 128 + ((k4 ^ (px & 7)) << 4);
      *reinterpret_cast<float4*>(sAh + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<float4*>(sAl + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    }
    fence_proxy_async_smem();                         // generic writes -> tensor-core reads
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_tf32(kStemPx, 64);
      const uint64_t ah = smem_desc_kmajor(smem_u32(sAh), 1024, 2);
      const uint64_t al = smem_desc_kmajor(smem_u32(sAl), 1024, 2);
      const uint64_t bh = smem_desc_kmajor(smem_u32(sBh), 1024, 2);
      const uint64_t bl = smem_desc_kmajor(smem_u32(sBl), 1024, 2);
      constexpr int kSteps = (9 * CIN + 7) / 8;        // K = 8 per MMA (+32 bytes)
#pragma unroll
      for (int ks = 0; ks < kSteps; ++ks) {
        mma_tf32(tmem, al + 2 * ks, bh + 2 * ks, idesc, ks > 0 ? 1u : 0u);
        mma_tf32(tmem, ah + 2 * ks, bl + 2 * ks, idesc, 1u);
      }
#pragma unroll
      for (int ks = 0; ks < kSteps; ++ks) mma_tf32(tmem, ah + 2 * ks, bh + 2 * ks, idesc, 1u);
      mma_commit(bar);
    }
    const bool ok_t = mbar_wait_bounded(bar, iter & 1, p.timeout);
    if (!ok_t && p.err) atomicOr(p.err, kErrTimeoutAcc);
    tc_fence_after();
    ok = __syncthreads_and(ok_t);
    if (!ok) break;
    // Thread = pixel = TMEM lane; BN once for the 64 channels.
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float x[64], v[64];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float a[32];
      tmem_ld32(lane_base + 32 * h, a);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        x[32 * h + j] = fmaf(a[j], sc[32 * h + j], bi[32 * h + j]);
        v[32 * h + j] = 0.f;
      }
    }
    tc_fence_before();                                // the next tile's MMAs overwrite TMEM
    const int nrows = min(R, p.OH - oh0);
    const int n16 = nrows * OW * 8;                   // 16-byte chunks of the tile's output
    for (int t = 0; t < p.T; ++t) {
      uint8_t* tile_s = smem + (t & 1) * kStemATile;  // the A tiles are free after the MMAs
      if (p.tma_out && t >= 2) {                      // this tile's store of t - 2 has read it
        if (tid == 0) bulk_wait_group_read<1>();
        __syncthreads();
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t bits = 0;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = 8 * q + 2 * u + e;
            if (neuron_step<MODE>(v[j], x[j], p.decay, p.tau, p.v_th, p.v_reset))
              bits |= 0x3C00u << (16 * e);
          }
          w[u] = bits;
        }
        *reinterpret_cast<uint4*>(tile_s + px * 128 + ((q ^ (px & 7)) << 4)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (p.tma_out) {
        // The tile (128-byte swizzled pixel rows) is the TMA box
        // {64 ch, OW, R rows}; rows past OH are not written.
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
          tma_store_5d(&p.tmap_out, tile_s, 0, 0, oh0, b, t);
          bulk_commit_group();
        }
        continue;
      }
      __syncthreads();
      uint4* dst = reinterpret_cast<uint4*>(
          p.out + ((static_cast<size_t>(t) * P + static_cast<size_t>(b) * p.OH * OW +
                    static_cast<size_t>(oh0) * OW) * 64));
      for (int i = tid; i < n16; i += kStemThreads) {
        const int pp = i >> 3, cg = i & 7;
        dst[i] = *reinterpret_cast<const uint4*>(tile_s + pp * 128 + ((cg ^ (pp & 7)) << 4));
      }
    }
  }
  if (p.tma_out && tid == 0) bulk_wait_group<0>();   // stores complete before the block exits
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// ------------------------------------------------ general tensor-core stem
// Dense stem of any kernel size and stride (K = Cin*KH*KW <= 192), up to 64
// output channels, input repeated over T (Tin = 1: one GEMM, the neuron runs
// T steps on it) or one frame per timestep (Tin = T: one GEMM per timestep,
// the membrane carried in registers), with a LIF/IF neuron or none (fp16 BN
// output).  A tile is R rows x TW columns of one image's output (TW =
// min(OW, 128), R = 128 / TW); a work unit is one tile and one GEMM (frame).
// GEMM: D[px][co] = im2col(x)[px][k] * w[co][k], M = 128 (TMEM lanes =
// pixels), K in 32-wide fp32 k-tiles, split into tf32 hi + lo parts on both
// sides (fp32-level accuracy): the resident weight k-tile holds the hi rows
// and then the lo rows, so ONE N = 128 MMA per 8-wide K step and A part
// gives x_a * [w_hi | w_lo]; two such MMAs (A = x_hi, x_lo) accumulate all
// four products, D[:, co] + D[:, 64 + co] being the full product.
//
// Two warp groups, so that the im2col work of one unit overlaps the
// epilogue of the previous one:
// * warps 0-7 (builders): the input window under a unit (every channel,
//   (R-1)*stride + KH rows, (TW-1)*stride + KW columns) arrives in one of two
//   staging buffers -- one TMA box requested two units ahead, by the
//   builders' thread 0 for the first two units and then by one epilogue
//   thread (fp32 rows with a 16-byte aligned pitch; the window's first
//   column sits dx in), or cp.async copies where the rows' pitch rules TMA
//   out; the builders expand
//   it into im2col k-tiles (hi/lo, a pixel's 32 columns split between two
//   threads) in a ring of two A stages, meet at a named barrier per k-tile,
//   and thread 0 then issues that k-tile's 8 MMAs into one of two TMEM
//   accumulators (128 columns each);
// * warps 8-15 (epilogue): thread = (pixel, 32 of the 64 channels); BN once,
//   neuron over T (or one step per frame, or the fp16 BN output); each
//   timestep's [pixels][Cout] fp16 tile is written into one of two shared
//   buffers; the two warps of a TMEM lane quarter (32 pixels, both channel
//   halves) meet at their own named barrier and send their 32 pixels by one
//   bulk copy: a tile's valid pixels are contiguous in the NHWC output
//   (R = 1: part of a row; R > 1: TW = OW, whole rows).  Bit-packed spikes
//   (p.bits_out) leave straight from registers as 16-bit words instead.
// 16 warps, 4 per SM sub-partition: 128 registers a thread.  Every wait is
// bounded; a group whose wait expires sets the error word and stops, and the
// group waiting on it then expires in turn.
constexpr int kStemGThreads = 16 * 32;
constexpr int kStemGBuild = 256;                // builder threads (warps 0-7)
constexpr int kStemGEpi0 = 8;                   // first epilogue warp (8-15)
constexpr int kStemGMaxK = 192;
constexpr int kStemGMaxStage = 20 * 1024;       // bytes of one staged input window (two alternate)
constexpr int kStemGOutBytes = 128 * 64 * 2;    // one timestep's output tile
__host__ __device__ constexpr int stem_tcg_stages(int nk) { return nk <= 5 ? 2 : 1; }
__host__ __device__ constexpr int stem_tcg_smem_bytes(int nk) {
  return 2 * nk * 8192 + stem_tcg_stages(nk) * 32768 + 2 * kStemGMaxStage + 2 * kStemGOutBytes +
         kStemGMaxK * 4 + 2 * 64 * 4 + 16 * 8 + 1024;
}
__host__ __device__ constexpr int stem_tcg_smem_max() {
  return stem_tcg_smem_bytes(5) > stem_tcg_smem_bytes(6) ? stem_tcg_smem_bytes(5)
                                                         : stem_tcg_smem_bytes(6);
}

// Two channels of the stem epilogue: the neuron step of each (membrane v[j],
// input x[j], tau = 2 input pre-halved) as fp16 spikes, or the fp16 BN output.
template <int MODE>
__device__ __forceinline__ uint32_t stem_pack2(float (&v)[32], const float (&x)[32], int j,
                                               const StemParams& p) {
  float2 f;
  if constexpr (MODE == kModeNone) {
    f = make_float2(x[j], x[j + 1]);
  } else {
    // Spikes as 0.0 / 1.0 floats, converted in pairs (exact).
    f.x = neuron_step<MODE>(v[j], x[j], p.decay, p.tau, p.v_th, p.v_reset) ? 1.f : 0.f;
    f.y = neuron_step<MODE>(v[j + 1], x[j + 1], p.decay, p.tau, p.v_th, p.v_reset) ? 1.f : 0.f;
  }
  const __half2 hv = __float22half2_rn(f);
  return *reinterpret_cast<const uint32_t*>(&hv);
}

// Dual output: two channels' neuron step on the fp16-rounded BN output
// (packed in `h2`), exactly as the standalone LIF node computes it from that
// stored tensor (tau = 2: the input halved), as fp16 spikes.
template <int MODE>
__device__ __forceinline__ uint32_t stem_spike2(float (&v)[32], uint32_t h2, int j,
                                                const StemParams& p) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
  const float a = MODE == kModeLifHalf ? f.x * 0.5f : f.x;
  const float b = MODE == kModeLifHalf ? f.y * 0.5f : f.y;
  float2 s2;
  s2.x = neuron_step<MODE>(v[j], a, p.decay, p.tau, p.v_th, p.v_reset) ? 1.f : 0.f;
  s2.y = neuron_step<MODE>(v[j + 1], b, p.decay, p.tau, p.v_th, p.v_reset) ? 1.f : 0.f;
  const __half2 hv = __float22half2_rn(s2);
  return *reinterpret_cast<const uint32_t*>(&hv);
}

// DUAL (MODE = the neuron): `out` gets the fp16 BN output and `out2` the
// spikes of MODE's neuron over T on it -- the stem and the standalone neuron
// node after it in one pass (MS-ResNet's stem and its first block's LIF).
template <int MODE, bool DUAL>
__global__ void __launch_bounds__(kStemGThreads, 1)
stem_tc_gen_kernel(const __grid_constant__ StemParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int K = p.Cin * p.KH * p.KW;
  const int nk = (K + 31) / 32;
  const int S = stem_tcg_stages(nk);
  const int TW = min(p.OW, 128), R = 128 / TW;
  const int IR = (R - 1) * p.stride + p.KH, IC = (TW - 1) * p.stride + p.KW;
  const int XP = p.in_pitch;                             // staged row pitch (floats)
  uint8_t* sB = smem;                                    // [nk][hi 64 ch, lo 64 ch][32] fp32, 128B swizzle
  uint8_t* sA = sB + nk * 16384;                         // [S][hi, lo][128 px][32]
  float* xs0 = reinterpret_cast<float*>(sA + S * 32768); // [2][Cin][IR][XP] staged input windows
  uint8_t* so = reinterpret_cast<uint8_t*>(xs0) + 2 * kStemGMaxStage;   // [2][4 quarters][32 px][Cout] fp16
  int* kofs = reinterpret_cast<int*>(so + 2 * kStemGOutBytes);
  float* sc = reinterpret_cast<float*>(kofs + kStemGMaxK);
  float* bi = sc + 64;
  uint64_t* a_empty = reinterpret_cast<uint64_t*>(bi + 64);   // [2] MMAs done with an A stage
  uint64_t* acc_full = a_empty + 2;                           // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;                         // [2] epilogue -> MMA
  uint64_t* in_full = acc_empty + 2;                          // [2] staged window landed (TMA)
  uint64_t* drain = in_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  // TMA windows: [0] requested by the builders' thread 0, [1] waited for by
  // the builders, [2] requested by the epilogue's window thread.
  int* win_state = reinterpret_cast<int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 256);
      mbar_init(&in_full[i], 1);
    }
    mbar_init(drain, 1);
    win_state[0] = win_state[1] = win_state[2] = 0;
    fence_mbar_init();
    if (p.tma_in) prefetch_tmap(&p.tmap_in);
  }
  if (warp == 0) { tmem_alloc(tmem_slot, 256); tmem_relinquish(); }
  // Resident weights (constant data): B[co][k] hi/lo, zero past Cout / K.
  for (int i = tid; i < nk * 64 * 32; i += kStemGThreads) {
    const int kt = i / 2048, rem = i - kt * 2048, co = rem >> 5, kk = rem & 31;
    const int k = kt * 32 + kk;
    const float wv = (co < p.Cout && k < K) ? __ldg(p.w + static_cast<size_t>(co) * K + k) : 0.f;
    const float hi = to_tf32(wv);
    *reinterpret_cast<float*>(sB + kt * 16384 + sw128_f32(co, kk)) = hi;
    *reinterpret_cast<float*>(sB + kt * 16384 + 8192 + sw128_f32(co, kk)) = wv - hi;
  }
  // Column k = (ci*KH + kh)*KW + kw (the [Cout][Cin][KH][KW] weight order)
  // reads staged element kofs[k] + (pixel row * stride) * XP + pixel col * stride.
  for (int k = tid; k < nk * 32; k += kStemGThreads) {
    if (k < K) {
      const int ci = k / (p.KH * p.KW), r = k - ci * p.KH * p.KW, kh = r / p.KW, kw = r - kh * p.KW;
      kofs[k] = (ci * IR + kh) * XP + kw;
    } else {
      kofs[k] = -1;                                      // padding column: zero
    }
  }
  if (tid < 64) {
    const bool cv = tid < p.Cout;
    // BN pre-scaled by 1/2 for the tau = 2 LIF step, as in the conv epilogues.
    // (DUAL: unscaled, the fp16 BN output is stored.)
    constexpr bool half_bn = MODE == kModeLifHalf && !DUAL;
    sc[tid] = cv ? (half_bn ? p.scale[tid] * 0.5f : p.scale[tid]) : 0.f;
    bi[tid] = cv ? (half_bn ? p.bias[tid] * 0.5f : p.bias[tid]) : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();                                            // input and output belong to the stream

  const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
  const int tiles_w = (p.OW + TW - 1) / TW, tiles_h = (p.OH + R - 1) / R;
  // 32-bit unit arithmetic: the host keeps B * tiles * frames below 2^31.
  const int n_tiles = p.B * tiles_h * tiles_w;
  const int n_gemm = p.Tin > 1 ? p.T : 1;
  // Units of this block: tile blockIdx.x + (u / n_gemm) * gridDim.x, GEMM
  // (frame) u % n_gemm, for u < n_units.
  const int bx = static_cast<int>(blockIdx.x), gx = static_cast<int>(gridDim.x);
  const int my_tiles = bx < n_tiles ? (n_tiles - 1 - bx) / gx + 1 : 0;
  const int n_units = my_tiles * n_gemm;
  // Unit cursor: unit u's GEMM g and tile (column wi, row hi, image b),
  // stepped one unit at a time with compares instead of divisions (the
  // kernel is issue-bound): the next unit is the next GEMM of the same tile,
  // or the first GEMM of the tile gx further on.
  struct UnitCursor { int g, wi, hi, b; };
  const int step_w = gx % tiles_w, step_r = gx / tiles_w;
  const int step_h = step_r % tiles_h, step_b = step_r / tiles_h;
  auto cursor_at_first = [&]() {
    UnitCursor c;
    const int rest = bx / tiles_w;
    c.g = 0;
    c.wi = bx - rest * tiles_w;
    c.b = rest / tiles_h;
    c.hi = rest - c.b * tiles_h;
    return c;
  };
  auto cursor_next = [&](UnitCursor& c) {
    if (++c.g < n_gemm) return;
    c.g = 0;
    c.wi += step_w;
    int cy = c.wi >= tiles_w;
    if (cy) c.wi -= tiles_w;
    c.hi += step_h + cy;
    cy = c.hi >= tiles_h;
    if (cy) c.hi -= tiles_h;
    c.b += step_b + cy;
  };
  // TMA input windows: unit u's window into buffer u & 1, its first column
  // rounded down to a 16-byte boundary (negative coordinates read zero).
  // The builders' thread 0 requests units 0 and 1; the window of unit u + 2
  // is requested by one epilogue thread once the MMAs of unit u are complete
  // (so every builder is done reading buffer u & 1), keeping the ~1k-cycle
  // issue off the builders' path.
  const uint32_t in_bytes = static_cast<uint32_t>(XP) * IR * p.Cin * 4;
  auto load_window = [&](const UnitCursor& c, int u) {
    const int iw0 = c.wi * TW * p.stride - p.pad;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&in_full[u & 1], in_bytes);
    tma_load_5d(xs0 + (u & 1) * (kStemGMaxStage / 4), &p.tmap_in, &in_full[u & 1], iw0 & ~3,
                c.hi * R * p.stride - p.pad, 0, c.b, c.g);
  };
  if (warp < kStemGEpi0) {
    // ------------------------------------------------ builders + MMA issue
    const int HW = p.H * p.W;
    const int px = tid & 127, half = tid >> 7;           // pixel; column half of each k-tile
    const int pr = px / TW, pc = px - (px / TW) * TW;    // pixel's row and column in the tile
    const int pofs = pr * p.stride * XP + pc * p.stride; // this pixel's window origin
    // cp.async (all builders): unit u's window, rows of pitch XP = IC.
    auto stage_window = [&](const UnitCursor& c, float* dst) {
      const int ih0 = c.hi * R * p.stride - p.pad, iw0 = c.wi * TW * p.stride - p.pad;
      const float* xin = p.x + (static_cast<size_t>(c.g) * p.B + c.b) * static_cast<size_t>(p.Cin) * HW;
      for (int row = warp; row < p.Cin * IR; row += kStemGBuild / 32) {
        const int ci = row / IR, ih = ih0 + row - ci * IR;
        const bool rv = ih >= 0 && ih < p.H;
        const float* src = xin + static_cast<size_t>(ci) * HW + static_cast<size_t>(rv ? ih : 0) * p.W;
#pragma unroll 4
        for (int cc = lane; cc < IC; cc += 32) {
          const int iw = iw0 + cc;
          const bool valid = rv && iw >= 0 && iw < p.W;
          cp_async4(dst + row * XP + cc, valid ? src + iw : p.x, valid);
        }
      }
      cp_async_commit();
    };
    const uint32_t idesc = idesc_tf32(128, 128);
    int kc = 0;                                          // k-tiles built so far (ring position)
    int requested = 0, waited = 0;                       // TMA windows (thread 0: the first two)
    bool ok = true, ok0 = true, issued = false;          // ok0, issued: thread 0 (MMA issuer)
    UnitCursor cur = cursor_at_first();                  // unit un
    if (n_units > 0) {
      if (!p.tma_in) stage_window(cur, xs0);
      else if (tid == 0) {
        load_window(cur, 0);
        UnitCursor c1 = cur;
        cursor_next(c1);
        if (n_units > 1) load_window(c1, 1);
        requested = min(n_units, 2);
      }
    }
    for (int un = 0; ok && un < n_units; ++un, cursor_next(cur)) {
      // Every builder passed the previous unit's last k-tile barrier, so the
      // buffer of unit un - 1 is free for unit un + 1.
      bool okw = true;
      if (p.tma_in) {
        okw = mbar_wait_bounded_sleep(&in_full[un & 1], static_cast<uint32_t>((un >> 1) & 1), p.timeout);
        waited = un + 1;
        if (!okw && p.err) atomicOr(p.err, kErrTimeoutFull);
      } else {
        if (un + 1 < n_units) {
          UnitCursor c1 = cur;
          cursor_next(c1);
          stage_window(c1, xs0 + ((un + 1) & 1) * (kStemGMaxStage / 4));
        }
        else cp_async_commit();                          // an empty group keeps the counting uniform
        cp_async_wait<1>();                              // this unit's window has landed
        named_barrier(1, kStemGBuild);
      }
      const int oh0 = cur.hi * R, ow0 = cur.wi * TW;
      const int iw0 = ow0 * p.stride - p.pad;
      const float* xs = xs0 + (un & 1) * (kStemGMaxStage / 4) + (p.tma_in ? iw0 - (iw0 & ~3) : 0);
      const bool pv = pr < R && oh0 + pr < p.OH && ow0 + pc < p.OW;
      const int a = un & 1;
      for (int kt = 0; kt < nk; ++kt, ++kc) {
        const int s = S == 2 ? (kc & 1) : 0;             // S is 1 or 2
        const int use = S == 2 ? (kc >> 1) : kc;
        bool okk = okw;
        if (okk && use > 0) {                            // the MMAs that read this stage are done
          okk = mbar_wait_bounded_sleep(&a_empty[s], static_cast<uint32_t>((use - 1) & 1), p.timeout);
          if (!okk && p.err) atomicOr(p.err, kErrTimeoutEmpty);
        }
        if (okk) {
          // This thread's 16 columns: their window offsets (4 vector loads),
          // then all 16 values, then the hi/lo split and the stores.
          int ko[16];
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            const int4 k4 = *reinterpret_cast<const int4*>(kofs + kt * 32 + half * 16 + c4 * 4);
            ko[4 * c4] = k4.x; ko[4 * c4 + 1] = k4.y; ko[4 * c4 + 2] = k4.z; ko[4 * c4 + 3] = k4.w;
          }
          float xv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) xv[j] = (pv && ko[j] >= 0) ? xs[ko[j] + pofs] : 0.f;
          uint8_t* ah = sA + s * 32768;
          uint8_t* al = ah + 16384;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            float hi[4], lo[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              hi[j] = to_tf32(xv[4 * c4 + j]);
              lo[j] = xv[4 * c4 + j] - hi[j];
            }
            const int chunk = half * 4 + c4;
            const int off = px * 128 + ((chunk ^ (px & 7)) << 4);
            *reinterpret_cast<float4*>(ah + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<float4*>(al + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
          }
        }
        fence_proxy_async_smem();                        // generic writes -> tensor-core reads
        if (named_barrier_or(1, kStemGBuild, !okk || !ok0)) { ok = false; break; }
        if (tid == 0) {
          if (kt == 0 && un >= 2) {                      // the epilogue has read this accumulator
            ok0 = mbar_wait_bounded_sleep(&acc_empty[a], static_cast<uint32_t>(((un >> 1) - 1) & 1),
                                          p.timeout);
            if (!ok0 && p.err) atomicOr(p.err, kErrTimeoutAccEmpty);
          }
          if (ok0) {
            tc_fence_after();
            const uint32_t acc = tmem + static_cast<uint32_t>(a * 128);
            uint8_t* ah = sA + s * 32768;
            const uint64_t dah = smem_desc_kmajor(smem_u32(ah), 1024, 2);
            const uint64_t dal = smem_desc_kmajor(smem_u32(ah + 16384), 1024, 2);
            const uint64_t db = smem_desc_kmajor(smem_u32(sB + kt * 16384), 1024, 2);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              mma_tf32(acc, dah + 2 * ks, db + 2 * ks, idesc, (kt > 0 || ks > 0) ? 1u : 0u);
              mma_tf32(acc, dal + 2 * ks, db + 2 * ks, idesc, 1u);
            }
            issued = true;
            mma_commit(&a_empty[s]);
            if (kt == nk - 1) mma_commit(&acc_full[a]);
          }
        }
      }
    }
    if (!p.tma_in) cp_async_wait<0>();
    if (tid == 0) {
      win_state[0] = requested;
      win_state[1] = waited;
      // Every MMA issued completes before TMEM is released.
      if (issued) {
        mma_commit(drain);
        if (!mbar_wait_bounded(drain, 0, p.timeout) && p.err) atomicOr(p.err, kErrTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------ epilogue
    const int q = warp & 3, h = (warp - kStemGEpi0) >> 2;   // TMEM lane quarter; channel half
    const int c0 = 32 * h;
    const int nch = max(0, min(32, p.Cout - c0)) / 8;    // 16-byte chunks this thread stores
    const bool lead = h == 0 && lane == 0;               // issues the quarter's bulk copies
    const int qbar = 2 + q;                              // the quarter's two warps
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int row_bytes = p.Cout * 2;
    const bool win_thread = p.tma_in && q == 0 && h == 1 && lane == 0;   // requests windows u + 2
    int win_req = 0;
    float v[32];
    uint32_t out_uses = 0;                               // timestep tiles written so far
    UnitCursor cur = cursor_at_first();                  // unit un
    for (int un = 0; un < n_units; ++un, cursor_next(cur)) {
      const int a = un & 1;
      const int g = cur.g;
      bool okw = true;
      if (lead) {
        okw = mbar_wait_bounded_sleep(&acc_full[a], static_cast<uint32_t>((un >> 1) & 1), p.timeout);
        if (!okw && p.err) atomicOr(p.err, kErrTimeoutAcc);
      }
      if (named_barrier_or(qbar, 64, !okw)) break;
      if (win_thread && un + 2 < n_units) {
        UnitCursor c2 = cur;
        cursor_next(c2);
        cursor_next(c2);
        load_window(c2, un + 2);
        win_req = un + 3;
      }
      tc_fence_after();
      float x[32];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {                   // 16 columns at a time
        uint32_t rh[16], rl[16];                         // x_a * w_hi and x_a * w_lo columns
        tmem_ld16_nowait(lane_base + static_cast<uint32_t>(a * 128 + c0 + 16 * hh), rh);
        tmem_ld16_nowait(lane_base + static_cast<uint32_t>(a * 128 + 64 + c0 + 16 * hh), rl);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          x[16 * hh + j] = __uint_as_float(rh[j]) + __uint_as_float(rl[j]);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);                        // this accumulator may be overwritten
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] = fmaf(x[j], sc[c0 + j], bi[c0 + j]);
      if (g == 0) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      const int b = cur.b, oh0 = cur.hi * R, ow0 = cur.wi * TW;
      const int npix = R == 1 ? min(TW, p.OW - ow0) : min(R, p.OH - oh0) * p.OW;
      const int nq = max(0, min(32, npix - 32 * q));     // this quarter's valid pixels
      const long long pix0 = (static_cast<long long>(b) * p.OH + oh0) * p.OW + ow0 + 32 * q;
      const int t_first = p.Tin > 1 ? g : 0, t_last = p.Tin > 1 ? g : p.T - 1;
      // One quarter's 32 pixel rows of a [pixels][Cout] fp16 tile; 128-byte
      // pixel rows put every lane's chunk c in one bank group, so those are
      // written in a lane-rotated order.
      auto write_tile = [&](uint8_t* ob, const uint32_t (&w)[16]) {
        uint8_t* orow = ob + lane * row_bytes + c0 * 2;
        if (row_bytes % 128 == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = (i + lane) & 3;
            if (c < nch) {
              uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3];
              if (c == 1) { w0 = w[4]; w1 = w[5]; w2 = w[6]; w3 = w[7]; }
              if (c == 2) { w0 = w[8]; w1 = w[9]; w2 = w[10]; w3 = w[11]; }
              if (c == 3) { w0 = w[12]; w1 = w[13]; w2 = w[14]; w3 = w[15]; }
              *reinterpret_cast<uint4*>(orow + 16 * c) = make_uint4(w0, w1, w2, w3);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (c < nch)
              *reinterpret_cast<uint4*>(orow + 16 * c) =
                  make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        }
      };
      if constexpr (DUAL) {
        // The unit's fp16 BN output tile (slot 0) is written once and sent
        // for each of its timesteps; the spike tile (slot 1) each timestep.
        uint32_t wx[16];
#pragma unroll
        for (int q2 = 0; q2 < 16; ++q2) {
          const __half2 hv = __float22half2_rn(make_float2(x[2 * q2], x[2 * q2 + 1]));
          wx[q2] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        uint8_t* ox = so + q * (kStemGOutBytes / 4);
        uint8_t* os = so + kStemGOutBytes + q * (kStemGOutBytes / 4);
        if (lead) bulk_wait_group_read<0>();             // the previous unit's copies read both
        named_barrier(qbar, 64);
        write_tile(ox, wx);
        for (int t = t_first; t <= t_last; ++t) {
          uint32_t w[16];
#pragma unroll
          for (int q2 = 0; q2 < 16; ++q2) w[q2] = 0u;
          if (nch == 4) {
#pragma unroll
            for (int q2 = 0; q2 < 16; ++q2) w[q2] = stem_spike2<MODE>(v, wx[q2], 2 * q2, p);
          } else {
#pragma unroll
            for (int q2 = 0; q2 < 8; ++q2) w[q2] = stem_spike2<MODE>(v, wx[q2], 2 * q2, p);
          }
          if (t > t_first) {                             // the last spike tile has been read
            if (lead) bulk_wait_group_read<0>();
            named_barrier(qbar, 64);
          }
          write_tile(os, w);
          fence_proxy_async_smem();                      // generic writes -> bulk-copy reads
          named_barrier(qbar, 64);
          if (lead) {
            if (nq > 0) {
              const size_t o = (static_cast<size_t>(t) * P + pix0) * p.Cout;
              bulk_store_1d(p.out + o, ox, static_cast<uint32_t>(nq) * row_bytes);
              bulk_store_1d(p.out2 + o, os, static_cast<uint32_t>(nq) * row_bytes);
            }
            bulk_commit_group();
          }
        }
      } else if (MODE != kModeNone && p.bits_out) {
        // Bit-packed spikes (SNN_FLAG_SPIKE_BITS), stored straight from
        // registers: this pixel's 32 (or 16) channels as u16 words, channel
        // c in bit c%16 of word c/16 -- a sixteenth of the fp16 tile.
        const int wn = p.Cout / 16;
        uint16_t* ob = reinterpret_cast<uint16_t*>(p.out) + (pix0 + lane) * wn + c0 / 16;
        for (int t = t_first; t <= t_last; ++t) {
          uint32_t m = 0;
          if (nch == 4) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              m |= neuron_step<MODE>(v[j], x[j], p.decay, p.tau, p.v_th, p.v_reset) ? 1u << j : 0u;
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              m |= neuron_step<MODE>(v[j], x[j], p.decay, p.tau, p.v_th, p.v_reset) ? 1u << j : 0u;
          }
          if (lane < nq && nch > 0) {
            uint16_t* o = ob + static_cast<size_t>(t) * P * wn;
            o[0] = static_cast<uint16_t>(m);
            if (nch == 4) o[1] = static_cast<uint16_t>(m >> 16);
          }
        }
      } else {
      for (int t = t_first; t <= t_last; ++t, ++out_uses) {
        uint32_t w[16];
        if (nch == 4) {
#pragma unroll
          for (int q2 = 0; q2 < 16; ++q2) w[q2] = stem_pack2<MODE>(v, x, 2 * q2, p);
        } else {                                         // 16 channels (Cout = 48) or none
#pragma unroll
          for (int q2 = 0; q2 < 8; ++q2) w[q2] = stem_pack2<MODE>(v, x, 2 * q2, p);
#pragma unroll
          for (int q2 = 8; q2 < 16; ++q2) w[q2] = 0u;
        }
        uint8_t* ob = so + (out_uses & 1) * kStemGOutBytes + q * (kStemGOutBytes / 4);
        // The bulk copy that last read this buffer (two tiles ago) is done reading.
        if (lead) bulk_wait_group_read<1>();
        named_barrier(qbar, 64);
        write_tile(ob, w);
        fence_proxy_async_smem();                        // generic writes -> bulk-copy reads
        named_barrier(qbar, 64);
        if (lead) {                                      // one group per timestep tile
          if (nq > 0)
            bulk_store_1d(p.out + (static_cast<size_t>(t) * P + pix0) * p.Cout, ob,
                          static_cast<uint32_t>(nq) * row_bytes);
          bulk_commit_group();
        }
      }
      }
    }
    if (lead) bulk_wait_group<0>();                      // stores complete before the block exits
    if (win_thread) win_state[2] = win_req;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      // Windows requested but not waited for (a stopped run) land before the
      // block exits.
      const int req = max(win_state[0], win_state[2]);
      for (int u = win_state[1]; u < req; ++u)
        mbar_wait_bounded_sleep(&in_full[u & 1], static_cast<uint32_t>((u >> 1) & 1), p.timeout);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------ elementwise neuron glue
// Fused Add + neuron and MaxPool + neuron over T (the reference's
// add_lif_fused_kernel and maxpool_lif_fused_kernel,
// sengine/kernels/add_lif_fused.py:19-75 and pool_lif_fused.py:15-79), with
// the neuron of the model (LIF v*(1-1/tau) + x/tau, or IF, hard reset).
// Memory-bound: thread = (output pixel, 8 channels), 16-byte loads and
// stores, membrane in registers across the T timesteps.
struct GlueParams {
  const __half* a;     // Add: [T][P][C]; MaxPool: input [T][B][H][W][C]
  const __half* b;     // Add: second input [T][P][C]
  __half* out;         // [T][B][OH][OW][C] spikes
  float* state;        // [B*OH*OW][C] membrane or null
  int T, B, H, W, C, OH, OW, KH, KW, stride, pad, flags;
  float tau, decay, v_th, v_reset;
};

template <int MODE>
__device__ __forceinline__ uint4 glue_neuron8(float (&v)[8], const float (&x)[8], const GlueParams& p) {
  if constexpr (MODE == kModeNone) {
    // No neuron (plain max pool): the inputs pass through (exact, they came from fp16).
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      w[u] = __half_as_ushort(__float2half_rn(x[2 * u])) |
             (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(x[2 * u + 1]))) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint32_t bits = 0;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 2 * u + e;
        // kModeLifHalf takes the input pre-halved (exact).
        const float xi = MODE == kModeLifHalf ? x[j] * 0.5f : x[j];
        if (neuron_step<MODE>(v[j], xi, p.decay, p.tau, p.v_th, p.v_reset)) bits |= 0x3C00u << (16 * e);
      }
      w[u] = bits;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// KS: compile-time square pool window (2 or 3: every window load is issued
// before the max, padding reads as -inf), or 0 for a runtime window.  I: the
// element index type, int wherever (pixels x 8-channel groups) fits (its
// divisions are several times cheaper than 64-bit ones), else long long.
template <int MODE, bool POOL, int KS = 0, typename I = long long>
__global__ void __launch_bounds__(256)
glue_neuron_kernel(const GlueParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int c8n = p.C / 8;
  const I P = static_cast<I>(p.B) * p.OH * p.OW;
  const I n = P * c8n;
  for (I idx = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
       idx += static_cast<I>(gridDim.x) * blockDim.x) {
    const I pix = idx / c8n;
    const int c8 = static_cast<int>(idx - pix * c8n);
    const size_t spix = static_cast<size_t>(pix);
    int ow = 0, oh = 0, b = 0;
    if constexpr (POOL) {
      const I r = pix / p.OW;
      ow = static_cast<int>(pix - r * p.OW);
      const I bb = r / p.OH;
      oh = static_cast<int>(r - bb * p.OH);
      b = static_cast<int>(bb);
    }
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = (MODE != kModeNone && (p.flags & kReadState)) ? p.state[spix * p.C + c8 * 8 + j] : 0.f;
    for (int t = 0; t < p.T; ++t) {
      float x[8];
      if constexpr (POOL && KS > 0) {
        const uint4 ninf4 = make_uint4(0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u);
        const __half* plane = p.a + (static_cast<size_t>(t) * p.B + b) * p.H * p.W * p.C;
        uint4 win[KS * KS];
#pragma unroll
        for (int kh = 0; kh < KS; ++kh) {
#pragma unroll
          for (int kw = 0; kw < KS; ++kw) {
            const int ih = oh * p.stride + kh - p.pad, iw = ow * p.stride + kw - p.pad;
            win[kh * KS + kw] = (ih >= 0 && ih < p.H && iw >= 0 && iw < p.W)
                ? __ldg(reinterpret_cast<const uint4*>(plane + (static_cast<size_t>(ih) * p.W + iw) * p.C) + c8)
                : ninf4;
          }
        }
        __half2 m[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) m[j] = reinterpret_cast<const __half2*>(&win[0])[j];
#pragma unroll
        for (int w = 1; w < KS * KS; ++w) {
#pragma unroll
          for (int j = 0; j < 4; ++j) m[j] = __hmax2(m[j], reinterpret_cast<const __half2*>(&win[w])[j]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(m[j]);
          x[2 * j] = f.x; x[2 * j + 1] = f.y;
        }
      } else if constexpr (POOL) {
        __half2 m[4];
        const __half2 ninf = __halves2half2(__ushort_as_half(0xFC00), __ushort_as_half(0xFC00));
#pragma unroll
        for (int j = 0; j < 4; ++j) m[j] = ninf;
        for (int kh = 0; kh < p.KH; ++kh) {
          const int ih = oh * p.stride + kh - p.pad;
          if (ih < 0 || ih >= p.H) continue;
          for (int kw = 0; kw < p.KW; ++kw) {
            const int iw = ow * p.stride + kw - p.pad;
            if (iw < 0 || iw >= p.W) continue;
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(
                p.a + (((static_cast<size_t>(t) * p.B + b) * p.H + ih) * p.W + iw) * p.C) + c8);
            const __half2* hv = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j) m[j] = __hmax2(m[j], hv[j]);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(m[j]);
          x[2 * j] = f.x; x[2 * j + 1] = f.y;
        }
      } else {
        // Add + neuron, or the neuron of one input alone when b is null.
        const size_t off = (static_cast<size_t>(t) * static_cast<size_t>(P) + spix) * p.C;
        const uint4 ua = __ldg(reinterpret_cast<const uint4*>(p.a + off) + c8);
        const uint4 ub = p.b ? __ldg(reinterpret_cast<const uint4*>(p.b + off) + c8)
                             : make_uint4(0, 0, 0, 0);
        const __half2* ha = reinterpret_cast<const __half2*>(&ua);
        const __half2* hb = reinterpret_cast<const __half2*>(&ub);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fa = __half22float2(ha[j]), fb = __half22float2(hb[j]);
          x[2 * j] = fa.x + fb.x;                      // exact: two fp16 values
          x[2 * j + 1] = fa.y + fb.y;
        }
      }
      reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(t) * static_cast<size_t>(P) + spix) * p.C)[c8] =
          glue_neuron8<MODE>(v, x, p);
    }
    if (MODE != kModeNone && (p.flags & kWriteState)) {
#pragma unroll
      for (int j = 0; j < 8; ++j) p.state[spix * p.C + c8 * 8 + j] = v[j];
    }
  }
}

// Plain max pool of bit-packed spikes (no neuron): the maximum of 0/1
// spikes is their OR, so thread = one output pixel of one of the T*B images
// ORs, word by word (16 channels each), the u16 words of its window
// (padding contributes nothing, as -inf never wins the max of a window
// holding a real pixel) and expands each word to 16 fp16 0/1 through a
// 16-entry nibble table in shared memory (two 16-byte stores).  a: the
// packed input [T*B][H][W][C/8] bytes; out: [T*B][OH][OW][C] fp16.
template <int KS>
__global__ void __launch_bounds__(256)
maxpool_bits_kernel(const GlueParams p) {
  __shared__ uint2 nib_lut[16];                          // nibble -> four fp16 (1.0 = 0x3C00)
  if (threadIdx.x < 16) {
    uint32_t h[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) h[b] = (threadIdx.x >> b) & 1u ? 0x3C00u : 0u;
    nib_lut[threadIdx.x] = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();
  // y: the T*B images; x: output pixels of one image, 32-bit (the host keeps
  // H*W*C/16 below 2^30).
  const int wn = p.C / 16;
  const int per_img = p.OH * p.OW;
  const int KH = KS > 0 ? KS : p.KH, KW = KS > 0 ? KS : p.KW;
  for (int img = blockIdx.y; img < p.T * p.B; img += gridDim.y) {
    const uint16_t* plane = reinterpret_cast<const uint16_t*>(p.a) + static_cast<size_t>(img) * p.H * p.W * wn;
    __half* out_img = p.out + static_cast<size_t>(img) * per_img * p.C;
    for (int pix = blockIdx.x * blockDim.x + threadIdx.x; pix < per_img; pix += gridDim.x * blockDim.x) {
      const int oh = pix / p.OW;
      const int ow = pix - oh * p.OW;
      uint4* dst = reinterpret_cast<uint4*>(out_img + static_cast<size_t>(pix) * p.C);
      for (int w = 0; w < wn; ++w) {
        uint32_t m = 0;
#pragma unroll
        for (int kh = 0; kh < KH; ++kh) {
          const int ih = oh * p.stride + kh - p.pad;
#pragma unroll
          for (int kw = 0; kw < KW; ++kw) {
            const int iw = ow * p.stride + kw - p.pad;
            if (ih >= 0 && ih < p.H && iw >= 0 && iw < p.W)
              m |= __ldg(plane + (ih * p.W + iw) * wn + w);
          }
        }
        const uint2 e0 = nib_lut[m & 15u], e1 = nib_lut[(m >> 4) & 15u];
        const uint2 e2 = nib_lut[(m >> 8) & 15u], e3 = nib_lut[(m >> 12) & 15u];
        dst[2 * w] = make_uint4(e0.x, e0.y, e1.x, e1.y);
        dst[2 * w + 1] = make_uint4(e2.x, e2.y, e3.x, e3.y);
      }
    }
  }
}

// ------------------------------------------------ timestep-split neuron scan
// Second phase of the timestep-split fused layer (snn_conv_forward_tsplit):
// the first phase ran the conv + BN for all T*B images at once (no neuron,
// fp32 BN output z); here thread = (pixel, channel) runs the neuron over T
// with the membrane in a register, adds the residual (after the neuron: the
// SEW add; before it: the neuron integrates bn + residual) and writes the
// fp16 spike.  The layers this form serves have few neurons per timestep (a
// 4x4x512 DVS stage-4 map is 32k), so a thread owns one, and the loads of
// kTsplitBatch timesteps are issued together before their neuron steps run:
// one HBM round trip for all of T <= 16.  The arithmetic is the fused
// epilogue's (for tau = 2 the input is halved exactly, as there), so the
// spikes equal the one-pass layer's for the same BN outputs.
struct TsplitParams {
  const float* z;          // [T][P][C] BN output
  const __half* residual;  // [T][P][C] or null
  __half* out;             // [T][P][C]
  float* state;            // [P][C] membrane or null
  long long P;             // pixels per timestep (B*OH*OW)
  int T, C, flags;
  float tau, decay, v_th, v_reset;
};
constexpr int kTsplitBatch = 16;

template <int MODE, int RM>
__global__ void __launch_bounds__(256)
tsplit_neuron_kernel(const TsplitParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const long long n = p.P * p.C;                           // neurons per timestep
  const size_t plane = static_cast<size_t>(n);
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const size_t base = static_cast<size_t>(idx);          // = pixel * C + channel
    float v = (p.flags & kReadState) ? p.state[base] : 0.f;
    for (int t0 = 0; t0 < p.T; t0 += kTsplitBatch) {
      float zb[kTsplitBatch];
      __half rb[kTsplitBatch];
#pragma unroll
      for (int j = 0; j < kTsplitBatch; ++j) {
        if (t0 + j < p.T) {
          const size_t off = static_cast<size_t>(t0 + j) * plane + base;
          zb[j] = __ldg(p.z + off);
          if constexpr (RM != kResNone) rb[j] = p.residual[off];
        }
      }
#pragma unroll
      for (int j = 0; j < kTsplitBatch; ++j) {
        if (t0 + j >= p.T) break;
        const float r = RM != kResNone ? __half2float(rb[j]) : 0.f;
        // kModeLifHalf takes bn/2 (exact), plus r/2 when the residual enters the neuron.
        float xi = MODE == kModeLifHalf ? zb[j] * 0.5f : zb[j];
        if constexpr (RM == kResAddBefore) xi = __fadd_rn(xi, MODE == kModeLifHalf ? r * 0.5f : r);
        const bool sp = neuron_step<MODE>(v, xi, p.decay, p.tau, p.v_th, p.v_reset);
        __half o;
        if constexpr (RM == kResAddAfter) o = __float2half_rn((sp ? 1.f : 0.f) + r);
        else o = __ushort_as_half(sp ? 0x3C00u : 0u);
        p.out[static_cast<size_t>(t0 + j) * plane + base] = o;
      }
    }
    if (p.flags & kWriteState) p.state[base] = v;
  }
}

// One block (1024 threads) per image.  Phase 1: thread (c8, slot) sums 8
// consecutive channels (16-byte loads) over every 16th (t, hw) position; the
// partial sums are combined in shared memory and scaled: feat = sum / HW / T
// (exact for the small-integer SEW activations).  Phase 2: a warp per four
// output classes, 16-byte weight loads.  dynamic smem = 17*C floats.
constexpr int kHeadSlots = 16;
__global__ void __launch_bounds__(1024)
head_pool_fc_kernel(const __half* __restrict__ x, const float* __restrict__ fc_w,
                    const float* __restrict__ fc_b, float* __restrict__ logits,
                    int T, int B, int HW, int C, int NC) {
  extern __shared__ float sm[];
  float* part = sm;                          // [kHeadSlots][C]
  float* feat = sm + kHeadSlots * C;         // [C]
  const int b = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const int c8n = C / 8;
  for (int task = threadIdx.x; task < c8n * kHeadSlots; task += blockDim.x) {
    const int c8 = task % c8n, slot = task / c8n;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // Position pos = t*HW + i stepped by kHeadSlots without divisions
    // (measured faster than a division per position: Spikformer head 38 ->
    // 34 us, SEW-ResNet-18 11.4 -> 10.1 us).
    int t = 0, i = slot;
    while (i >= HW) { i -= HW; ++t; }
#pragma unroll 4
    for (int pos = slot; pos < T * HW; pos += kHeadSlots) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(
          x + ((static_cast<size_t>(t) * B + b) * HW + i) * C) + c8);
      i += kHeadSlots;
      while (i >= HW) { i -= HW; ++t; }
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        s[2 * j] += f.x; s[2 * j + 1] += f.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) part[slot * C + c8 * 8 + j] = s[j];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int sl = 0; sl < kHeadSlots; ++sl) acc += part[sl * C + c];
    feat[c] = acc / static_cast<float>(HW) / static_cast<float>(T);
  }
  __syncthreads();
  // Phase 2: with more classes than warps, a warp takes four at a time, so
  // four rows' weight loads (and their reductions) are in flight together
  // (SEW-ResNet's 100 classes: 15 -> 10 us); up to one class per warp, one.
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  constexpr int kCls = 4;
  const int cls = NC > nwarps ? kCls : 1;
  for (int n0 = warp * cls; n0 < NC; n0 += nwarps * cls) {
    float acc[kCls];
#pragma unroll
    for (int u = 0; u < kCls; ++u) acc[u] = 0.f;
#pragma unroll 2
    for (int c4 = lane; c4 < C / 4; c4 += 32) {
      const float4 f = *reinterpret_cast<const float4*>(feat + 4 * c4);
#pragma unroll
      for (int u = 0; u < kCls; ++u) {
        if (u < cls && n0 + u < NC) {
          const float4 w = __ldg(reinterpret_cast<const float4*>(fc_w + static_cast<size_t>(n0 + u) * C) + c4);
          acc[u] = fmaf(f.x, w.x, fmaf(f.y, w.y, fmaf(f.z, w.z, fmaf(f.w, w.w, acc[u]))));
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
      for (int u = 0; u < kCls; ++u)
        if (u < cls) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], off);   // cls: warp-uniform
    }
    if (lane == 0) {
#pragma unroll
      for (int u = 0; u < kCls; ++u)
        if (u < cls && n0 + u < NC) logits[static_cast<size_t>(b) * NC + n0 + u] = acc[u] + (fc_b ? fc_b[n0 + u] : 0.f);
    }
  }
}

}  // namespace snn
