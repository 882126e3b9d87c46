// Spikformer spiking self-attention core fused with its attention LIF, for
// sm_100a.
//
// Per (timestep t, image b, head h), with q, k, v the head's spike rows
// [N tokens][HD]:
//     x = (q k^T * scale) v,   spikes = LIF_{v_th}(x) over t
// (reference models/spikformer.py:122-127 and the fused op it becomes,
// sengine/tdl/attention_ops.py:50-82).  Products of spikes are integer
// counts, so (q k^T) v == q (k^T v) exactly in fp32, and the kernel computes
// the latter -- two small GEMMs on the tensor cores, every operand brought in
// by TMA straight from the [T*B][N][C] activations:
//
//   GEMM 1  D1[e][d] = sum_m k[m][e] v[m][d]   (M = 64 >= HD, N = HD, K = tokens)
//           A = k tile, B = v tile, both MN-major (token rows of the head's HD
//           channels; rows past N zero-filled).  D1 rows >= HD are unused.
//   GEMM 2  D2[n][d] = sum_e q[n][e] D1[e][d]  (M = 128 tokens per tile, N = HD, K = HD)
//           A = q tile, K-major; B = D1 as fp16 (integers <= N: exact), written
//           row e = channel into shared memory, MN-major.
//
// D2 lives in TMEM with lane = token and column = channel, so each epilogue
// thread owns one token's HD membranes for all T timesteps and writes its
// spikes as whole 64/128-byte rows.  One CTA per (image, head) takes the
// timesteps in passes of kAttnTC; thread 0 issues the TMA loads and MMAs,
// warps 0..HD/16-1 turn D1 into the GEMM-2 operand, warp w reads GEMM-2
// lane quarter w%4 of M-tile w/4.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include "snn_ptx.cuh"

namespace snn {

constexpr int kAttnThreads = 256;
constexpr int kAttnMaxN = 256;              // two 128-token M-tiles, one token per thread
constexpr int kAttnTC = 2;                  // timesteps per pass

struct AttnParams {
  CUtensorMap tmap_q;        // 3-D {C, N, T*B} fp16, box {HD, min(N,128), 1}
  CUtensorMap tmap_k;        // 3-D {C, N, T*B} fp16, box {HD, kv_rows, 1}
  CUtensorMap tmap_v;
  __half* out;               // [T*B][N][C] spikes
  float* state;              // [B][N][C] membrane or null
  unsigned* err;
  int T, B, N, heads, C, flags;
  int kv_rows;               // N rounded up to 16 (GEMM-1 K extent)
  int lif_half;              // tau == 2: folded two-FMA update
  float scale, decay, tau, v_th, v_reset;
  unsigned long long timeout;
};

template <int HD>
struct AttnCfg {
  static constexpr int kRowB = HD * 2;                  // bytes of one token's head slice
  static constexpr int kLayout = HD == 32 ? 4 : 2;      // SWIZZLE_64B / SWIZZLE_128B
  static constexpr int kSbo = 8 * kRowB;                // 8-row group
  static constexpr int kQTile = 128 * kRowB;            // one 128-token M-tile of q
  static constexpr int kKVTile = kAttnMaxN * kRowB;     // k or v rows of one timestep
  static constexpr int kDTile = HD * kRowB;             // D1 as fp16, HD rows
  static constexpr int kStep = kAttnTC * (2 * kQTile + 2 * kKVTile + kDTile);
  static constexpr int kSmemBytes = kStep + 64 + 1024;
  // TMEM: D2 of (u, m) at columns (2u + m) * HD; D1 of u at u * HD (consumed
  // before the GEMM-2 MMAs overwrite it).
  static constexpr int kTmemCols = 2 * kAttnTC * HD;
  static_assert(kTmemCols == 128 || kTmemCols == 256, "TMEM allocation must be a power of 2");
};

// Byte offset of 16-byte chunk c of row r in a swizzled tile of kRowB rows.
template <int HD>
__device__ __forceinline__ int attn_swz(int r, int c) {
  if constexpr (HD == 32) return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
  else return r * 128 + ((c ^ (r & 7)) << 4);
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, HD == 32 ? 2 : 1)
spikformer_attn_lif_kernel(const __grid_constant__ AttnParams p) {
  using Cfg = AttnCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                                          // [u][m]
  uint8_t* sK = sQ + kAttnTC * 2 * Cfg::kQTile;                // [u]
  uint8_t* sV = sK + kAttnTC * Cfg::kKVTile;                   // [u]
  uint8_t* sD = sV + kAttnTC * Cfg::kKVTile;                   // [u] D1 as fp16
  uint64_t* bar_kv = reinterpret_cast<uint64_t*>(smem + Cfg::kStep);
  uint64_t* bar_q = bar_kv + 1;
  uint64_t* bar_g1 = bar_kv + 2;
  uint64_t* bar_g2 = bar_kv + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_kv + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int b = blockIdx.x / p.heads, h = blockIdx.x % p.heads;
  const int N = p.N, C = p.C;
  const int n_mt = (N + 127) / 128;
  const int q_rows = min(N, 128);

  if (tid == 0) {
    mbar_init(bar_kv, 1);
    mbar_init(bar_q, 1);
    mbar_init(bar_g1, 1);
    mbar_init(bar_g2, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&p.tmap_q);
    prefetch_tmap(&p.tmap_k);
    prefetch_tmap(&p.tmap_v);
  }
  if (warp == 0) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();                            // q, k, v, state and out belong to the stream

  // Epilogue identity: GEMM-2 lane quarter warp%4 of M-tile warp/4.
  const int mt = warp >> 2;
  const int tok = mt * 128 + (warp & 3) * 32 + lane;
  const bool tok_ok = tok < N;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  const size_t state_row = (static_cast<size_t>(b) * N + tok) * C + h * HD;
  float vm[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d)
    vm[d] = ((p.flags & kReadState) && tok_ok) ? p.state[state_row + d] : 0.f;

  // GEMM 1: M = 64 (rows >= HD unused), N = HD, A and B MN-major.
  const uint32_t idesc1 = idesc_f16_major(64, HD, true, true);
  // GEMM 2: M = 128, N = HD, A K-major, B MN-major.
  const uint32_t idesc2 = idesc_f16_major(128, HD, false, true);
  constexpr uint32_t kKStep = (2 * Cfg::kSbo) >> 4;           // 16 rows along K, descriptor units
  const int n_pass = (p.T + kAttnTC - 1) / kAttnTC;
  // Loads of a pass (thread 0).  k/v tiles are refilled as soon as GEMM 1 of
  // the previous pass has completed and q tiles as soon as GEMM 2 has, so the
  // next pass's loads overlap this pass's conversion and epilogue.
  int kv_issued = 0, q_issued = 0;
  auto issue_kv = [&](int ps) {
    const int tcn_ = min(kAttnTC, p.T - ps * kAttnTC);
    mbar_arrive_expect_tx(bar_kv, tcn_ * 2 * p.kv_rows * Cfg::kRowB);
    for (int u = 0; u < tcn_; ++u) {
      const int tb = (ps * kAttnTC + u) * p.B + b;
      tma_load_3d(sK + u * Cfg::kKVTile, &p.tmap_k, bar_kv, h * HD, 0, tb);
      tma_load_3d(sV + u * Cfg::kKVTile, &p.tmap_v, bar_kv, h * HD, 0, tb);
    }
    ++kv_issued;
  };
  auto issue_q = [&](int ps) {
    const int tcn_ = min(kAttnTC, p.T - ps * kAttnTC);
    mbar_arrive_expect_tx(bar_q, tcn_ * n_mt * q_rows * Cfg::kRowB);
    for (int u = 0; u < tcn_; ++u)
      for (int m = 0; m < n_mt; ++m)
        tma_load_3d(sQ + (2 * u + m) * Cfg::kQTile, &p.tmap_q, bar_q, h * HD, m * 128,
                    (ps * kAttnTC + u) * p.B + b);
    ++q_issued;
  };
  if (tid == 0) { issue_kv(0); issue_q(0); }
  bool stop = false;
  for (int pass = 0; pass < n_pass && !stop; ++pass) {
    const int t0 = pass * kAttnTC;
    const int tcn = min(kAttnTC, p.T - t0);
    const uint32_t ph = pass & 1;
    if (tid == 0) {
      // GEMM 1 per timestep, K = 16 tokens per MMA.
      if (!mbar_wait_bounded(bar_kv, ph, p.timeout)) {
        atomicOr(p.err, kErrTimeoutFull);
        *abort_flag = 1;
      } else {
        tc_fence_after();
        for (int u = 0; u < tcn; ++u) {
          // A: rows of HD channels; a 64-row M reads its second half one
          // 8-row group further (inside the tile; those D1 rows are unused).
          const uint64_t a_desc = smem_desc_mnmajor(smem_u32(sK + u * Cfg::kKVTile), Cfg::kSbo,
                                                    Cfg::kSbo, Cfg::kLayout);
          const uint64_t b_desc = smem_desc_mnmajor(smem_u32(sV + u * Cfg::kKVTile), Cfg::kSbo,
                                                    Cfg::kSbo, Cfg::kLayout);
          for (int ks = 0; ks < p.kv_rows / 16; ++ks)
            mma_f16(tmem + u * HD, a_desc + ks * kKStep, b_desc + ks * kKStep, idesc1,
                    ks > 0 ? 1u : 0u);
        }
      }
      mma_commit(bar_g1);                // arrives at once when nothing was issued
    }
    // D1 -> fp16 GEMM-2 operand: row e (= channel) holds D1[e][0..HD).  An
    // M = 64 accumulator keeps rows 16q..16q+15 in lanes 32q..32q+15.
    if (warp < HD / 16) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_g1, ph, p.timeout));
      tc_fence_after();
      if (ok && tid == 0 && pass + 1 < n_pass) issue_kv(pass + 1);   // k/v tiles are free
      if (ok) {
        const int e = 16 * warp + lane;
        for (int u = 0; u < tcn; ++u) {
#pragma unroll
          for (int c0 = 0; c0 < HD; c0 += 32) {
            float a[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + u * HD + c0, a);
            if (lane < 16) {
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const __half2 hv = __floats2half2_rn(a[8 * c + 2 * i], a[8 * c + 2 * i + 1]);
                  w[i] = *reinterpret_cast<const uint32_t*>(&hv);
                }
                *reinterpret_cast<uint4*>(sD + u * Cfg::kDTile + attn_swz<HD>(e, c0 / 8 + c)) =
                    make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
        }
      } else {
        if (lane == 0) atomicOr(p.err, kErrTimeoutAcc);
        *abort_flag = 1;
      }
      fence_proxy_async_smem();          // generic-proxy writes -> tensor-core reads
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (*abort_flag) {
        // a wait above gave up: issue nothing
      } else if (!mbar_wait_bounded(bar_q, ph, p.timeout)) {
        atomicOr(p.err, kErrTimeoutFull);
        *abort_flag = 1;
      } else {
        for (int u = 0; u < tcn; ++u) {
          const uint64_t b_desc = smem_desc_mnmajor(smem_u32(sD + u * Cfg::kDTile), Cfg::kSbo,
                                                    Cfg::kSbo, Cfg::kLayout);
          for (int m = 0; m < n_mt; ++m) {
            const uint64_t a_desc = smem_desc_kmajor(smem_u32(sQ + (2 * u + m) * Cfg::kQTile),
                                                     Cfg::kSbo, Cfg::kLayout);
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks)   // A: +32 bytes along the row; B: +16 rows
              mma_f16(tmem + (2 * u + m) * HD, a_desc + 2 * ks, b_desc + ks * kKStep, idesc2,
                      ks > 0 ? 1u : 0u);
          }
        }
      }
      mma_commit(bar_g2);
    }
    bool fail = !mbar_wait_bounded(bar_g2, ph, p.timeout);
    if (fail) atomicOr(p.err, kErrTimeoutAcc);
    tc_fence_after();
    fail = __syncthreads_or(fail || *abort_flag);
    if (fail) { stop = true; break; }
    if (tid == 0 && pass + 1 < n_pass) issue_q(pass + 1);            // q tiles are free
    if (mt < n_mt) {
      for (int u = 0; u < tcn; ++u) {
        float x[HD];
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 32) {
          float a[32];
          tmem_ld32(lane_base + (2 * u + mt) * HD + c0, a);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c0 + i] = a[i];
        }
        uint32_t packed[HD / 2];
#pragma unroll
        for (int d = 0; d < HD; d += 2) {
          bool s[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float xs = x[d + i] * p.scale;   // exact: a multiple of scale
            float hv;
            if (p.lif_half) hv = fmaf(vm[d + i], 0.5f, xs * 0.5f);
            else hv = __fadd_rn(__fmul_rn(vm[d + i], p.decay), __fdiv_rn(xs, p.tau));
            s[i] = hv >= p.v_th;
            vm[d + i] = s[i] ? p.v_reset : hv;
          }
          packed[d / 2] = (s[0] ? 0x3C00u : 0u) | (s[1] ? 0x3C000000u : 0u);
        }
        if (tok_ok) {
          uint4* o = reinterpret_cast<uint4*>(
              p.out + (static_cast<size_t>((t0 + u) * p.B + b) * N + tok) * C + h * HD);
#pragma unroll
          for (int j = 0; j < HD / 8; ++j)
            o[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();                     // TMEM and tiles free for the next pass
  }
  if (stop && tid == 0) {
    // Let loads still in flight land before the CTA's shared memory goes away.
    if (!mbar_wait_bounded(bar_kv, (kv_issued - 1) & 1, p.timeout) ||
        !mbar_wait_bounded(bar_q, (q_issued - 1) & 1, p.timeout))
      atomicOr(p.err, kErrTimeoutDrain);
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
