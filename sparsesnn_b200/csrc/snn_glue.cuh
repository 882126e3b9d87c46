// Memory-bound glue around the fused sparse layers of an SNN ResNet:
//  * stem_rows_kernel / stem_conv_lif_kernel: dense direct conv (small Cin,
//    e.g. RGB) + BN + LIF/IF over T, computed once when the input is
//    repeated over T (direct encoding) and written as fp16 NHWC spikes per
//    timestep (row-tiled fast path for 3x3 / 64-channel stems; the general
//    kernel covers other shapes and per-timestep inputs).
//  * head_pool_fc_kernel: global average pool + mean over T + linear head.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include "snn_conv.cuh"

namespace snn {

struct StemParams {
  const float* x;      // [Tin][B][Cin][H][W] fp32
  const float* w;      // [Cout][Cin][KH][KW] fp32
  const float* scale;  // [Cout]
  const float* bias;   // [Cout]
  __half* out;         // [T][B][OH][OW][Cout]
  int T, Tin, B, Cin, H, W, Cout, KH, KW, stride, pad, OH, OW, neuron;
  float tau, decay, v_th, v_reset;
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

// Row-tiled stem for the direct-encoding case (input repeated over T) of a
// 3x3 stride-1 pad-1 conv with 64 output channels on images at most 128
// pixels wide.  A block computes R = 128 / OW whole output rows of one image:
//  * the zero-padded input rows (CIN x (R+2) x (OW+2)), the weights
//    ([tap][64] fp32) and BN scale/bias are staged in shared memory;
//  * 256 threads: warp w computes pixels 32*(w/2) + lane of the block and
//    output channels 32*(w%2) .. +31 (weight reads are warp-wide broadcasts,
//    input reads consecutive words);
//  * BN once, then LIF/IF over T in registers; each timestep's spikes go to
//    a [128 px][64 ch] fp16 tile (128-byte rows, 16-byte chunks XOR-ed with
//    px & 7) and leave as fully coalesced 16-byte stores, since the block's
//    output rows are contiguous in the NHWC tensor.  Two tiles alternate, so
//    one barrier per timestep suffices.
constexpr int kStemPx = 128;
constexpr int kStemThreads = 256;

// Shared-memory layout of stem_rows_kernel, in floats: input rows, then the
// weights (16-byte aligned for float4 reads), scale, bias; the spike tiles
// start at stem_rows_smem_floats (128-byte aligned).
__host__ __device__ constexpr int stem_rows_ws_offset(int cin, int R, int OW) {
  return (cin * (R + 2) * (OW + 2) + 31) / 32 * 32;
}
__host__ __device__ constexpr int stem_rows_smem_floats(int cin, int R, int OW) {
  return (stem_rows_ws_offset(cin, R, OW) + 9 * cin * 64 + 128 + 31) / 32 * 32;
}

template <int CIN, int MODE>
__global__ void __launch_bounds__(kStemThreads)
stem_rows_kernel(const StemParams p) {
  extern __shared__ __align__(128) float sm[];
  const int OW = p.OW, R = kStemPx / OW, OWp = OW + 2;
  const int HWp = (R + 2) * OWp;
  const int bpi = (p.OH + R - 1) / R;                 // blocks per image
  const int b = blockIdx.x / bpi, oh0 = (blockIdx.x % bpi) * R;
  float* xs = sm;                                     // [CIN][R+2][OW+2]
  float* ws = sm + stem_rows_ws_offset(CIN, R, OW);   // [9*CIN][64], 16-byte aligned
  float* sc = ws + 9 * CIN * 64;                      // [64]
  float* bi = sc + 64;                                // [64]
  uint8_t* tiles = reinterpret_cast<uint8_t*>(sm + stem_rows_smem_floats(CIN, R, OW));
  const int tid = threadIdx.x;
  for (int i = tid; i < 9 * CIN * 64; i += kStemThreads) {
    const int co = i / (9 * CIN), k = i - co * (9 * CIN);   // source [Cout][Cin][3][3]
    ws[k * 64 + co] = p.w[i];
  }
  if (tid < 64) { sc[tid] = p.scale[tid]; bi[tid] = p.bias[tid]; }
  pdl_launch_dependents();
  pdl_wait();                                         // input and output belong to the stream
  const float* xin = p.x + static_cast<size_t>(b) * CIN * p.H * p.W;
  for (int i = tid; i < CIN * HWp; i += kStemThreads) {
    const int ci = i / HWp, rem = i - ci * HWp;
    const int r = rem / OWp, c = rem - r * OWp;
    const int ih = oh0 - 1 + r, iw = c - 1;
    xs[i] = (ih >= 0 && ih < p.H && iw >= 0 && iw < p.W)
                ? __ldg(xin + (static_cast<size_t>(ci) * p.H + ih) * p.W + iw) : 0.f;
  }
  __syncthreads();

  const int warp = tid / 32, lane = tid % 32;
  const int pxl = (warp >> 1) * 32 + lane;            // pixel within the block
  const int ch0 = (warp & 1) * 32;
  const int r = pxl / OW, c = pxl - (pxl / OW) * OW;
  const bool in_tile = pxl < R * OW;
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = 0.f;
  if (in_tile) {
#pragma unroll
    for (int ci = 0; ci < CIN; ++ci) {
#pragma unroll
      for (int kh = 0; kh < 3; ++kh) {
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
          const float xv = xs[ci * HWp + (r + kh) * OWp + c + kw];
          const float4* wr = reinterpret_cast<const float4*>(ws + ((ci * 3 + kh) * 3 + kw) * 64 + ch0);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 w4 = wr[q];
            acc[4 * q + 0] = fmaf(xv, w4.x, acc[4 * q + 0]);
            acc[4 * q + 1] = fmaf(xv, w4.y, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(xv, w4.z, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(xv, w4.w, acc[4 * q + 3]);
          }
        }
      }
    }
  }
  // BN output (pre-scaled by 1/2 for the tau = 2 LIF step, as in the conv epilogues).
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float s = MODE == kModeLifHalf ? sc[ch0 + j] * 0.5f : sc[ch0 + j];
    const float o = MODE == kModeLifHalf ? bi[ch0 + j] * 0.5f : bi[ch0 + j];
    acc[j] = fmaf(acc[j], s, o);
    v[j] = 0.f;
  }
  const int nrows = min(R, p.OH - oh0);
  const int n16 = nrows * OW * 8;                     // 16-byte chunks of the block's output
  const long long P = static_cast<long long>(p.B) * p.OH * OW;
  for (int t = 0; t < p.T; ++t) {
    uint8_t* tile = tiles + (t & 1) * (kStemPx * 128);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint32_t bits = 0;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = 8 * q + 2 * u + e;
          if (neuron_step<MODE>(v[j], acc[j], p.decay, p.tau, p.v_th, p.v_reset))
            bits |= 0x3C00u << (16 * e);
        }
        w[u] = bits;
      }
      const int cg = (ch0 >> 3) + q;
      *reinterpret_cast<uint4*>(tile + pxl * 128 + ((cg ^ (pxl & 7)) << 4)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
    __syncthreads();
    uint4* dst = reinterpret_cast<uint4*>(
        p.out + ((static_cast<size_t>(t) * P + static_cast<size_t>(b) * p.OH * OW +
                  static_cast<size_t>(oh0) * OW) * 64));
    for (int i = tid; i < n16; i += kStemThreads) {
      const int px = i >> 3, cg = i & 7;
      dst[i] = *reinterpret_cast<const uint4*>(tile + px * 128 + ((cg ^ (px & 7)) << 4));
    }
  }
}

// One block (1024 threads) per image.  Phase 1: thread (c8, slot) sums 8
// consecutive channels (16-byte loads) over every 16th (t, hw) position; the
// partial sums are combined in shared memory and scaled: feat = sum / HW / T
// (exact for the small-integer SEW activations).  Phase 2: one warp per
// output class, 16-byte weight loads.  dynamic smem = 17*C floats.
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
    for (int pos = slot; pos < T * HW; pos += kHeadSlots) {
      const int t = pos / HW, i = pos - t * HW;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(
          x + ((static_cast<size_t>(t) * B + b) * HW + i) * C) + c8);
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
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  for (int n = warp; n < NC; n += nwarps) {
    const float4* wr = reinterpret_cast<const float4*>(fc_w + static_cast<size_t>(n) * C);
    float acc = 0.f;
    for (int c4 = lane; c4 < C / 4; c4 += 32) {
      const float4 w = __ldg(wr + c4);
      const float4 f = *reinterpret_cast<const float4*>(feat + 4 * c4);
      acc = fmaf(f.x, w.x, fmaf(f.y, w.y, fmaf(f.z, w.z, fmaf(f.w, w.w, acc))));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) logits[static_cast<size_t>(b) * NC + n] = acc + (fc_b ? fc_b[n] : 0.f);
  }
}

}  // namespace snn
