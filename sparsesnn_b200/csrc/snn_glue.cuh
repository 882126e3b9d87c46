// Memory-bound glue around the fused sparse layers of an SNN ResNet:
//  * stem_conv_lif_kernel: dense direct conv (small Cin, e.g. RGB) + BN +
//    LIF/IF over T, computed once when the input is repeated over T
//    (direct encoding) and written as fp16 NHWC spikes per timestep.
//  * head_pool_fc_kernel: global average pool + mean over T + linear head.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

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

// One thread = one output pixel x 8 consecutive output channels; a block of
// 256 threads covers 256/(Cout/8) pixels.  Weights are staged in shared
// memory as [k][cout] (dynamic smem = K*Cout floats, K = Cin*KH*KW); each
// timestep's 8 spikes leave as one 16-byte store.
__global__ void __launch_bounds__(256)
stem_conv_lif_kernel(const StemParams p) {
  extern __shared__ float ws[];
  const int K = p.KH * p.KW * p.Cin;
  for (int i = threadIdx.x; i < K * p.Cout; i += blockDim.x) {
    const int k = i / p.Cout, co = i - k * p.Cout;
    // k = (ci*KH + kh)*KW + kw, matching the [Cout][Cin][KH][KW] source.
    ws[i] = p.w[static_cast<size_t>(co) * K + k];
  }
  __syncthreads();
  const int groups = p.Cout / 8;
  const int px_per_block = blockDim.x / groups;
  const int g = threadIdx.x % groups;
  const long long pix = static_cast<long long>(blockIdx.x) * px_per_block + threadIdx.x / groups;
  const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
  if (threadIdx.x >= px_per_block * groups || pix >= P) return;
  const int ow = static_cast<int>(pix % p.OW);
  const int oh = static_cast<int>((pix / p.OW) % p.OH);
  const int b = static_cast<int>(pix / (static_cast<long long>(p.OW) * p.OH));
  const int c0 = g * 8;
  float sc[8], bi[8], v[8], xb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) { sc[j] = p.scale[c0 + j]; bi[j] = p.bias[c0 + j]; v[j] = 0.f; xb[j] = 0.f; }
  for (int t = 0; t < p.T; ++t) {
    if (t == 0 || p.Tin > 1) {
      const float* xin = p.x + (static_cast<size_t>(p.Tin > 1 ? t : 0) * p.B + b) *
                                   static_cast<size_t>(p.Cin) * p.H * p.W;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      int k = 0;
      for (int ci = 0; ci < p.Cin; ++ci) {
        for (int kh = 0; kh < p.KH; ++kh) {
          const int ih = oh * p.stride + kh - p.pad;
          for (int kw = 0; kw < p.KW; ++kw, ++k) {
            const int iw = ow * p.stride + kw - p.pad;
            if (ih < 0 || ih >= p.H || iw < 0 || iw >= p.W) continue;
            const float xv = __ldg(xin + (static_cast<size_t>(ci) * p.H + ih) * p.W + iw);
            const float4 w0 = *reinterpret_cast<const float4*>(ws + k * p.Cout + c0);
            const float4 w1 = *reinterpret_cast<const float4*>(ws + k * p.Cout + c0 + 4);
            acc[0] = fmaf(xv, w0.x, acc[0]); acc[1] = fmaf(xv, w0.y, acc[1]);
            acc[2] = fmaf(xv, w0.z, acc[2]); acc[3] = fmaf(xv, w0.w, acc[3]);
            acc[4] = fmaf(xv, w1.x, acc[4]); acc[5] = fmaf(xv, w1.y, acc[5]);
            acc[6] = fmaf(xv, w1.z, acc[6]); acc[7] = fmaf(xv, w1.w, acc[7]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) xb[j] = fmaf(acc[j], sc[j], bi[j]);
    }
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      uint32_t bits = 0;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float h;
        if (p.neuron == 0) h = __fadd_rn(__fmul_rn(v[j + u], p.decay), __fdiv_rn(xb[j + u], p.tau));
        else h = __fadd_rn(v[j + u], xb[j + u]);
        const bool s = (h - p.v_th) >= 0.f;
        v[j + u] = s ? p.v_reset : h;
        bits |= (s ? 0x3C00u : 0u) << (16 * u);
      }
      packed[j / 2] = bits;
    }
    *reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(t) * P + pix) * p.Cout + c0) =
        make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

// One block per image: feat[c] = mean_t mean_hw x[t][b][hw][c];
// logits[b][n] = feat . fc_w[n] + fc_b[n].  dynamic smem = C floats.
__global__ void head_pool_fc_kernel(const __half* __restrict__ x, const float* __restrict__ fc_w,
                                    const float* __restrict__ fc_b, float* __restrict__ logits,
                                    int T, int B, int HW, int C, int NC) {
  extern __shared__ float feat[];
  const int b = blockIdx.x;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float tsum = 0.f;
    for (int t = 0; t < T; ++t) {
      const __half* xt = x + (static_cast<size_t>(t) * B + b) * static_cast<size_t>(HW) * C + c;
      float s = 0.f;
      for (int i = 0; i < HW; ++i) s += __half2float(xt[static_cast<size_t>(i) * C]);
      tsum += s / static_cast<float>(HW);
    }
    feat[c] = tsum / static_cast<float>(T);
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  for (int n = warp; n < NC; n += nwarps) {
    const float* wr = fc_w + static_cast<size_t>(n) * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s = fmaf(feat[c], wr[c], s);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) logits[static_cast<size_t>(b) * NC + n] = s + (fc_b ? fc_b[n] : 0.f);
  }
}

}  // namespace snn
