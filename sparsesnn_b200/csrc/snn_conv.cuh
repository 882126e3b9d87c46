// Fused 2:4-sparse implicit-GEMM Conv/Linear + BN + LIF/IF (+SEW add) over T
// timesteps for sm_100a.
//
// GEMM view (per CTA):  D[cout, pixel] = W_sp[cout, k] * X[k, pixel]
//   A = compressed 2:4 weights (M = 128 output channels), K-major, 64B swizzle
//   B = activations (N = BN output pixels per timestep), K-major, 128B swizzle;
//       one 64-channel slice of one filter tap per k-block, fetched by TMA from
//       the NHWC input with out-of-bounds zero fill providing the conv padding
//   D = FP32 accumulators in tensor memory, one BN-column block per timestep,
//       so each weight k-block is staged once and used for all T timesteps
//   E = 2:4 metadata, held in tensor memory for the CTA's whole K range
//
// Warp roles (6 warps): 0 = TMA producer, 1 = TMEM owner + MMA issuer,
// 2..5 = metadata loader + epilogue (BN, LIF recurrence over T with the
// membrane in registers, spike (+residual) store, final membrane store).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include "snn_ptx.cuh"

namespace snn {

constexpr int kBM = 128;             // output channels per CTA (UMMA M)
constexpr int kBN = 64;              // output pixels per timestep per CTA (UMMA N)
constexpr int kTC = 4;               // timesteps per accumulator chunk
constexpr int kStages = 5;           // smem pipeline depth
constexpr int kKB = 64;              // logical K per k-block (one 128B activation row)
constexpr int kABytes = kBM * (kKB / 2) * 2;     // 8 KB compressed weights
constexpr int kBBytes = kBN * kKB * 2;           // 8 KB activations per timestep
constexpr int kStageBytes = kABytes + kTC * kBBytes;
constexpr int kAccCols = kTC * kBN;              // 256 TMEM columns of accumulators
constexpr int kMetaCol = kAccCols;               // metadata columns start here
constexpr int kTmemCols = 512;
constexpr int kMaxMetaCols = kTmemCols - kMetaCol;  // => K <= 8192
constexpr int kThreads = 192;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;

enum NeuronKind : int { kLIF = 0, kIF = 1, kNoNeuron = 2 };
enum ConvFlags : int { kReadState = 1, kWriteState = 2 };
enum ErrCode : unsigned { kErrTimeoutFull = 1u, kErrTimeoutEmpty = 2u, kErrTimeoutAcc = 4u,
                          kErrTimeoutMeta = 8u, kErrTimeoutAccEmpty = 16u, kErrTimeoutDrain = 32u };

struct ConvParams {
  CUtensorMap tmap_a;        // compressed weights [Fpad][K/2] fp16
  CUtensorMap tmap_b[4];     // activations, one map per (h,w) stride parity
  const uint32_t* meta;      // [Fpad/128][K/32][128]
  const float* scale;        // [F]
  const float* bias;         // [F]
  float* state;              // [B*OH*OW][F] or null
  const __half* residual;    // [T*B*OH*OW][F] or null
  void* out;                 // [T*B*OH*OW][F] fp16 spikes, or fp32 BN output
  unsigned* err;             // device error word
  int F, Cin, KW, stride, pad;
  int n_kb, cin_blocks;      // k-blocks, 64-channel slices per tap
  int B, OH, OW, T;
  int tw, th, tn;            // tile extent (output coords) along w, h, image
  int tiles_w, tiles_h;      // tile grid (tiles_n implied by gridDim.x)
  int box_bytes;             // bytes one activation TMA box delivers (tw*th*tn*128)
  int neuron, flags;
  float decay, tau, v_th, v_reset;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ int floordiv2(int d) { return (d - (d & 1)) / 2; }

__global__ void __launch_bounds__(kThreads, 1)
fused_sparse_conv_lif_kernel(const __grid_constant__ ConvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                                   // kStages x kABytes
  uint8_t* sB = smem + kStages * kABytes;               // kStages x kTC x kBBytes
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* meta_ready = acc_empty + 1;
  uint64_t* drain = meta_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // Tile coordinates.
  const int tile = blockIdx.x;
  const int tw_i = tile % p.tiles_w;
  const int th_i = (tile / p.tiles_w) % p.tiles_h;
  const int tn_i = tile / (p.tiles_w * p.tiles_h);
  const int w0 = tw_i * p.tw, h0 = th_i * p.th, n0 = tn_i * p.tn;
  const int m_tile = blockIdx.y;
  const int n_chunks = (p.T + kTC - 1) / kTC;
  const int n_meta = 2 * p.n_kb;                        // sparse K steps (32 each)

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
    mbar_init(meta_ready, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmap_a);
    for (int i = 0; i < (p.stride == 2 ? 4 : 1); ++i) prefetch_tmap(&p.tmap_b[i]);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0; uint32_t phase = 0;
      int issued = 0;
      for (int c = 0; c < n_chunks && !*abort_flag; ++c) {
        const int t0 = c * kTC;
        const int tcn = min(kTC, p.T - t0);
        for (int kb = 0; kb < p.n_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutEmpty); *abort_flag = 1; break;
          }
          if (*abort_flag) break;
          mbar_arrive_expect_tx(&full[stage], kABytes + tcn * p.box_bytes);
          tma_load_2d(sA + stage * kABytes, &p.tmap_a, &full[stage], kb * (kKB / 2),
                      m_tile * kBM);
          const int tap = kb / p.cin_blocks;
          const int cb = kb - tap * p.cin_blocks;
          const int kh = tap / p.KW, kw = tap - kh * p.KW;
          int map = 0, hoff = kh - p.pad, woff = kw - p.pad;
          if (p.stride == 2) {
            const int hp = hoff & 1, wp = woff & 1;
            map = hp * 2 + wp;
            hoff = floordiv2(hoff); woff = floordiv2(woff);
          }
          for (int t = 0; t < tcn; ++t) {
            tma_load_4d(sB + (stage * kTC + t) * kBBytes, &p.tmap_b[map], &full[stage],
                        cb * kKB, w0 + woff, h0 + hoff, (t0 + t) * p.B + n0);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
      // Let every load already issued land before the CTA can exit.
      const int n_wait = min(issued, kStages);
      for (int i = 0; i < n_wait; ++i) {
        // Stage of the i-th most recent issue and the parity of that phase.
        const int back = issued - 1 - i;
        const int s = back % kStages;
        const uint32_t ph = (back / kStages) & 1;
        if (!mbar_wait_bounded(&full[s], ph, p.timeout_ns)) atomicOr(p.err, kErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, kBN, true);
      bool ok = mbar_wait_bounded(meta_ready, 0, p.timeout_ns);
      if (!ok) { atomicOr(p.err, kErrTimeoutMeta); *abort_flag = 1; }
      tc_fence_after();
      int stage = 0; uint32_t phase = 0;
      for (int c = 0; c < n_chunks && !*abort_flag; ++c) {
        const int tcn = min(kTC, p.T - c * kTC);
        if (c > 0) {
          if (!mbar_wait_bounded(acc_empty, (c - 1) & 1, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutAccEmpty); *abort_flag = 1; break;
          }
          tc_fence_after();
        }
        for (int kb = 0; kb < p.n_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutFull); *abort_flag = 1; break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * kABytes);
          const uint32_t b_base = smem_u32(sB + stage * kTC * kBBytes);
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const uint32_t ecol = kMetaCol + 2 * kb + s;
            const uint32_t e_addr = tmem + (ecol & ~1u);
            const uint32_t id = idesc | (ecol & 1u);
            const uint64_t adesc = smem_desc_kmajor(a_base + 32 * s, 512, 4);
            for (int t = 0; t < tcn; ++t) {
              const uint64_t bdesc = smem_desc_kmajor(b_base + t * kBBytes + 64 * s, 1024, 2);
              mma_sp_f16(tmem + t * kBN, adesc, bdesc, e_addr, id, (kb > 0 || s > 0) ? 1u : 0u);
            }
          }
          mma_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        mma_commit(acc_full);
      }
      // Drain: every MMA issued so far completes before TMEM is released.
      mma_commit(drain);
      if (!mbar_wait_bounded(drain, 0, p.timeout_ns)) atomicOr(p.err, kErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------- metadata + epilogue
    const int q = warp & 3;                      // TMEM lane quarter of this warp
    const int row = q * 32 + lane;               // output channel within the tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    {
      const uint32_t* src = p.meta + (static_cast<size_t>(m_tile) * n_meta) * kBM + row;
      int j = 0;
      for (; j + 8 <= n_meta; j += 8) {
        uint32_t r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = __ldg(src + static_cast<size_t>(j + i) * kBM);
        tmem_st8(lane_base + kMetaCol + j, r);
      }
      for (; j < n_meta; j += 8) {   // tail: store a full x8 group, padding with 0x44444444
        uint32_t r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          r[i] = (j + i < n_meta) ? __ldg(src + static_cast<size_t>(j + i) * kBM) : 0x44444444u;
        tmem_st8(lane_base + kMetaCol + j, r);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(meta_ready);
    }

    const int cout = m_tile * kBM + row;
    const bool cvalid = cout < p.F;
    const float sc = cvalid ? p.scale[cout] : 0.f;
    const float bi = cvalid ? p.bias[cout] : 0.f;
    const size_t P = static_cast<size_t>(p.B) * p.OH * p.OW;
    const int tile_px = p.tw * p.th;

    float v[kBN / 32][32];
    // Pixel index of each column (or -1 when outside the tensor).
    auto pixel_of = [&](int col) -> long long {
      const int dn = col / tile_px;
      const int rem = col - dn * tile_px;
      const int dh = rem / p.tw;
      const int dw = rem - dh * p.tw;
      const int n = n0 + dn, oh = h0 + dh, ow = w0 + dw;
      if (dn >= p.tn || n >= p.B || oh >= p.OH || ow >= p.OW) return -1;
      return (static_cast<long long>(n) * p.OH + oh) * p.OW + ow;
    };

#pragma unroll
    for (int g = 0; g < kBN / 32; ++g) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float v0 = 0.f;
        if ((p.flags & kReadState) && cvalid) {
          const long long px = pixel_of(g * 32 + i);
          if (px >= 0) v0 = p.state[px * p.F + cout];
        }
        v[g][i] = v0;
      }
    }

    for (int c = 0; c < n_chunks; ++c) {
      const int t0 = c * kTC;
      const int tcn = min(kTC, p.T - t0);
      if (*abort_flag) break;
      if (!mbar_wait_bounded(acc_full, c & 1, p.timeout_ns)) {
        atomicOr(p.err, kErrTimeoutAcc); *abort_flag = 1; break;
      }
      tc_fence_after();
      for (int t = 0; t < tcn; ++t) {
#pragma unroll
        for (int g = 0; g < kBN / 32; ++g) {
          float acc[32];
          tmem_ld32(lane_base + t * kBN + g * 32, acc);   // warp-collective: no early exit above
          const size_t tbase = static_cast<size_t>(t0 + t) * P;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const long long px = pixel_of(g * 32 + i);
            if (px < 0 || !cvalid) continue;
            const size_t o = (tbase + px) * p.F + cout;
            const float x = fmaf(acc[i], sc, bi);
            if (p.neuron == kNoNeuron) {
              static_cast<float*>(p.out)[o] = x;
              continue;
            }
            // Reference order: v*(1-1/tau) + x/tau, each op rounded (no FMA).
            float h;
            if (p.neuron == kLIF) h = __fadd_rn(__fmul_rn(v[g][i], p.decay), __fdiv_rn(x, p.tau));
            else h = __fadd_rn(v[g][i], x);
            const bool spike = (h - p.v_th) >= 0.f;
            v[g][i] = spike ? p.v_reset : h;
            float y = spike ? 1.f : 0.f;
            if (p.residual) y += __half2float(p.residual[o]);
            static_cast<__half*>(p.out)[o] = __float2half_rn(y);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
    }

    if ((p.flags & kWriteState) && cvalid && !*abort_flag) {
#pragma unroll
      for (int g = 0; g < kBN / 32; ++g) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const long long px = pixel_of(g * 32 + i);
          if (px >= 0) p.state[px * p.F + cout] = v[g][i];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace snn
