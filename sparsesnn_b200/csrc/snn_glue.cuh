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

// block = (64 output channels, 4 pixels); dynamic smem = 64 * KH*KW*Cin floats.
__global__ void stem_conv_lif_kernel(const StemParams p) {
  extern __shared__ float ws[];
  const int K = p.KH * p.KW * p.Cin;
  const int c_base = blockIdx.y * 64;
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  for (int i = tid; i < 64 * K; i += blockDim.x * blockDim.y) {
    const int cl = i / K, k = i - cl * K;
    const int co = c_base + cl;
    ws[i] = co < p.Cout ? p.w[static_cast<size_t>(co) * K + k] : 0.f;
  }
  __syncthreads();
  const int cout = c_base + threadIdx.x;
  const long long pix = static_cast<long long>(blockIdx.x) * blockDim.y + threadIdx.y;
  const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
  if (cout >= p.Cout || pix >= P) return;
  const int ow = static_cast<int>(pix % p.OW);
  const int oh = static_cast<int>((pix / p.OW) % p.OH);
  const int b = static_cast<int>(pix / (static_cast<long long>(p.OW) * p.OH));
  const float sc = p.scale[cout], bi = p.bias[cout];
  const float* wr = ws + threadIdx.x * K;
  float v = 0.f, x_bn = 0.f;
  for (int t = 0; t < p.T; ++t) {
    if (t == 0 || p.Tin > 1) {
      const float* xb = p.x + (static_cast<size_t>(p.Tin > 1 ? t : 0) * p.B + b) *
                                  static_cast<size_t>(p.Cin) * p.H * p.W;
      float acc = 0.f;
      for (int ci = 0; ci < p.Cin; ++ci) {
        for (int kh = 0; kh < p.KH; ++kh) {
          const int ih = oh * p.stride + kh - p.pad;
          if (ih < 0 || ih >= p.H) continue;
          for (int kw = 0; kw < p.KW; ++kw) {
            const int iw = ow * p.stride + kw - p.pad;
            if (iw < 0 || iw >= p.W) continue;
            acc = fmaf(xb[(static_cast<size_t>(ci) * p.H + ih) * p.W + iw],
                       wr[(ci * p.KH + kh) * p.KW + kw], acc);
          }
        }
      }
      x_bn = fmaf(acc, sc, bi);
    }
    float h;
    if (p.neuron == 0) h = __fadd_rn(__fmul_rn(v, p.decay), __fdiv_rn(x_bn, p.tau));
    else h = __fadd_rn(v, x_bn);
    const bool s = (h - p.v_th) >= 0.f;
    v = s ? p.v_reset : h;
    p.out[(static_cast<size_t>(t) * P + pix) * p.Cout + cout] = __float2half_rn(s ? 1.f : 0.f);
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
