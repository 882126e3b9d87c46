// Spikformer spiking self-attention core fused with its attention LIF, for
// sm_100a.
//
// Per (timestep t, image b, head h), with q, k, v the head's binary spike
// rows [N tokens][HD]:
//     x = (q k^T * scale) v,   spikes = LIF_{v_th}(x) over t
// (reference models/spikformer.py:122-127 and the fused op it becomes,
// sengine/tdl/attention_ops.py:50-82).  Every product of spikes is an
// integer, so (q k^T) v == q (k^T v) exactly in fp32: the kernel forms the
// small HD x HD matrix k^T v on the CUDA cores (bit masks and popcounts over
// the token axis) and multiplies q by it on the tensor cores:
//
//   A = q, one 128-token M-tile per MMA, TMA-loaded straight from the
//       [T*B][N][C] activations (64/128-byte rows of the head's HD channels,
//       rows past N zero-filled), K-major with 64B (HD=32) / 128B (HD=64)
//       swizzle;
//   B = (k^T v)^T as fp16 (integers <= N, exact), written K-major into shared
//       memory in the same swizzled layout;
//   D = fp32 in TMEM, lane = token, column = channel: each epilogue thread
//       owns one token's HD membranes for all T timesteps and writes its
//       spikes as whole 64/128-byte rows.
//
// One CTA per (image, head) walks t = 0..T-1; 8 warps: thread i builds the
// masks of token i; thread 0 issues the TMA loads and the MMAs; warp w reads
// accumulator lane quarter w%4 of M-tile w/4.
#pragma once
#include <cstdint>
#include <type_traits>
#include <cuda.h>
#include <cuda_fp16.h>
#include "snn_ptx.cuh"

namespace snn {

constexpr int kAttnThreads = 256;
constexpr int kAttnMaxN = 256;              // two 128-token M-tiles, one token per thread
constexpr unsigned kErrNonBinary = 128u;    // device error bit: q/k/v not all 0/1

struct AttnParams {
  CUtensorMap tmap_q;        // q as 3-D {C, N, T*B} fp16, box {HD, 128, 1}
  const __half* k;           // [T*B][N][C]
  const __half* v;
  __half* out;               // [T*B][N][C] spikes
  float* state;              // [B][N][C] membrane or null
  unsigned* err;
  int T, B, N, heads, C, flags;
  int lif_half;              // tau == 2: folded two-FMA update
  float scale, decay, tau, v_th, v_reset;
  unsigned long long timeout;
};

template <int HD>
struct AttnCfg {
  static constexpr int kRowB = HD * 2;                  // bytes of one token's head slice
  static constexpr int kLayout = HD == 32 ? 4 : 2;      // SWIZZLE_64B / SWIZZLE_128B
  static constexpr int kSbo = 8 * kRowB;
  static constexpr int kQTile = 128 * kRowB;
  static constexpr int kMaskWords = kAttnMaxN / 32;     // per channel
  static constexpr int kTmemCols = HD == 32 ? 64 : 128; // two accumulators of HD columns
  static constexpr int kSmemBytes =
      2 * kQTile + HD * kRowB + 2 * HD * kMaskWords * 4 + 64 + 1024;
};

// Byte offset of 16-byte chunk c of row r in a K-major swizzled tile.
template <int HD>
__device__ __forceinline__ int attn_swz(int r, int c) {
  if constexpr (HD == 32) return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
  else return r * 128 + ((c ^ (r & 7)) << 4);
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads)
spikformer_attn_lif_kernel(const __grid_constant__ AttnParams p) {
  using Cfg = AttnCfg<HD>;
  using Mask = typename std::conditional<HD == 32, uint32_t, unsigned long long>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                                          // 2 M-tiles
  uint8_t* sKV = sQ + 2 * Cfg::kQTile;                         // (k^T v)^T, HD rows
  uint32_t* sKm = reinterpret_cast<uint32_t*>(sKV + HD * Cfg::kRowB);   // [HD][words]
  uint32_t* sVm = sKm + HD * Cfg::kMaskWords;
  uint64_t* bar_q = reinterpret_cast<uint64_t*>(sVm + HD * Cfg::kMaskWords);
  uint64_t* bar_mma = bar_q + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int b = blockIdx.x / p.heads, h = blockIdx.x % p.heads;
  const int N = p.N, C = p.C;
  const int n_mt = (N + 127) / 128;
  const int n_words = (N + 31) / 32;

  if (tid == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_mma, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&p.tmap_q);
  }
  if (warp == 0) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_launch_dependents();
  pdl_wait();                            // q, k, v, state and out belong to the stream

  // Epilogue identity: accumulator lane quarter warp%4 of M-tile warp/4.
  const int mt = warp >> 2;
  const int tok = mt * 128 + (warp & 3) * 32 + lane;
  const bool tok_ok = tok < N;
  const uint32_t acc_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + mt * HD;
  const size_t state_row = (static_cast<size_t>(b) * N + tok) * C + h * HD;
  float vm[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d)
    vm[d] = ((p.flags & kReadState) && tok_ok) ? p.state[state_row + d] : 0.f;

  const uint32_t idesc = idesc_f16(128, HD, false);
  bool stop = false;
  for (int t = 0; t < p.T && !stop; ++t) {
    const int tb = t * p.B + b;
    // q tiles of this timestep (the previous step's MMAs are complete).
    // The box holds min(N, 128) rows; rows past N read as zero, rows past
    // the box are never stored.
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_q, n_mt * min(N, 128) * Cfg::kRowB);
      for (int m = 0; m < n_mt; ++m)
        tma_load_3d(sQ + m * Cfg::kQTile, &p.tmap_q, bar_q, h * HD, m * 128, tb);
    }
    // Bit masks of k and v over the token axis: word w of channel e holds
    // tokens 32w..32w+31 (thread = token).
    Mask kb = 0, vb = 0;
    bool bad = false;
    if (tid < N) {
      const size_t row = (static_cast<size_t>(tb) * N + tid) * C + h * HD;
      const uint4* kr = reinterpret_cast<const uint4*>(p.k + row);
      const uint4* vr = reinterpret_cast<const uint4*>(p.v + row);
#pragma unroll
      for (int j = 0; j < HD / 8; ++j) {
        const uint4 kx = __ldg(kr + j), vx = __ldg(vr + j);
        const uint32_t kw[4] = {kx.x, kx.y, kx.z, kx.w}, vw[4] = {vx.x, vx.y, vx.z, vx.w};
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t kh = (kw[u >> 1] >> (16 * (u & 1))) & 0xFFFFu;
          const uint32_t vh = (vw[u >> 1] >> (16 * (u & 1))) & 0xFFFFu;
          // 0x0000 / 0x8000 = zero, 0x3C00 = one; anything else is not a spike.
          const bool k1 = (kh & 0x7FFFu) != 0, v1 = (vh & 0x7FFFu) != 0;
          bad |= (k1 && kh != 0x3C00u) || (v1 && vh != 0x3C00u);
          kb |= static_cast<Mask>(k1) << (8 * j + u);
          vb |= static_cast<Mask>(v1) << (8 * j + u);
        }
      }
    }
    if (bad) atomicOr(p.err, kErrNonBinary);
#pragma unroll
    for (int e = 0; e < HD; ++e) {
      const uint32_t km = __ballot_sync(0xffffffffu, static_cast<uint32_t>((kb >> e) & 1));
      const uint32_t vmk = __ballot_sync(0xffffffffu, static_cast<uint32_t>((vb >> e) & 1));
      if (lane == (e & 31)) {
        sKm[e * Cfg::kMaskWords + warp] = km;
        sVm[e * Cfg::kMaskWords + warp] = vmk;
      }
    }
    __syncthreads();
    // (k^T v)^T[d][e] = #tokens with k[e] and v[d], as fp16 (exact: <= N).
    for (int idx = tid; idx < HD * HD / 2; idx += kAttnThreads) {
      const int d = idx / (HD / 2), e = 2 * (idx % (HD / 2));
      int s0 = 0, s1 = 0;
      for (int w = 0; w < n_words; ++w) {
        const uint32_t vw = sVm[d * Cfg::kMaskWords + w];
        s0 += __popc(sKm[e * Cfg::kMaskWords + w] & vw);
        s1 += __popc(sKm[(e + 1) * Cfg::kMaskWords + w] & vw);
      }
      *reinterpret_cast<__half2*>(sKV + attn_swz<HD>(d, e >> 3) + (e & 7) * 2) =
          __halves2half2(__int2half_rn(s0), __int2half_rn(s1));
    }
    fence_proxy_async_smem();            // generic-proxy writes -> tensor-core reads
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (!mbar_wait_bounded(bar_q, t & 1, p.timeout)) {
        atomicOr(p.err, kErrTimeoutFull);
        *abort_flag = 1;
      } else {
        const uint64_t b_desc = smem_desc_kmajor(smem_u32(sKV), Cfg::kSbo, Cfg::kLayout);
        for (int m = 0; m < n_mt; ++m) {
          const uint64_t a_desc =
              smem_desc_kmajor(smem_u32(sQ + m * Cfg::kQTile), Cfg::kSbo, Cfg::kLayout);
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks)   // K = 16 per MMA: +32 bytes along the row
            mma_f16(tmem + m * HD, a_desc + 2 * ks, b_desc + 2 * ks, idesc, ks > 0 ? 1u : 0u);
        }
      }
      mma_commit(bar_mma);               // arrives at once when nothing was issued
    }
    bool fail = !mbar_wait_bounded(bar_mma, t & 1, p.timeout);
    if (fail) atomicOr(p.err, kErrTimeoutAcc);
    tc_fence_after();
    fail = __syncthreads_or(fail || *abort_flag);
    if (fail) { stop = true; break; }
    if (mt < n_mt) {
      float x[HD];
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 32) {
        float a[32];
        tmem_ld32(acc_addr + c0, a);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[c0 + i] = a[i];
      }
      uint32_t packed[HD / 2];
#pragma unroll
      for (int d = 0; d < HD; d += 2) {
        bool s[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float xs = x[d + u] * p.scale;   // exact: a multiple of scale
          float hv;
          if (p.lif_half) hv = fmaf(vm[d + u], 0.5f, xs * 0.5f);
          else hv = __fadd_rn(__fmul_rn(vm[d + u], p.decay), __fdiv_rn(xs, p.tau));
          s[u] = hv >= p.v_th;
          vm[d + u] = s[u] ? p.v_reset : hv;
        }
        packed[d / 2] = (s[0] ? 0x3C00u : 0u) | (s[1] ? 0x3C000000u : 0u);
      }
      if (tok_ok) {
        uint4* o = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(tb) * N + tok) * C + h * HD);
#pragma unroll
        for (int j = 0; j < HD / 8; ++j)
          o[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
      }
    }
    tc_fence_before();
    __syncthreads();                     // TMEM, q and k^T v tiles free for the next step
  }
  if (!stop && (p.flags & kWriteState) && tok_ok) {
#pragma unroll
    for (int d = 0; d < HD; ++d) p.state[state_row + d] = vm[d];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace snn
