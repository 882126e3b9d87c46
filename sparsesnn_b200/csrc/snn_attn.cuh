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
// Persistent, warp-specialised pipeline over steps = (work item (b, h), t):
//   warp 12     TMA producer: k, v and q tiles of a step into a ring slot;
//   warp 13     MMA issuer + TMEM owner: GEMM 1 of step i, then GEMM 2 of
//               step i-1 (whose D1 operand is ready by then);
//   warps 8..   (HD/16 of them) D1 (TMEM, double-buffered) -> fp16 operand
//               in the step's slot;
//   warps 0..7  epilogue: D2 (TMEM, double-buffered) lane = token, column =
//               channel; each thread owns one token's HD membranes over the
//               item's T steps and writes its spikes as whole rows.
// All waits are bounded; a wait that gives up sets the device error word and
// an abort flag the other roles poll.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include "snn_ptx.cuh"

namespace snn {

constexpr int kAttnMaxN = 256;              // two 128-token M-tiles, one token per thread
constexpr int kAttnEpiWarps = 8;
constexpr int kAttnCvtWarp0 = 8;            // converter warps 8 .. 8 + HD/16 - 1 (lane quarters 0..)
constexpr int kAttnTmaWarp = 12;
constexpr int kAttnMmaWarp = 13;
constexpr int kAttnThreads = 14 * 32;

struct AttnParams {
  CUtensorMap tmap_q;        // 3-D {C, N, T*B} fp16, box {HD, min(N,128), 1}
  CUtensorMap tmap_k;        // 3-D {C, N, T*B} fp16, box {HD, kv_rows, 1}
  CUtensorMap tmap_v;
  CUtensorMap tmap_out;      // head_dim 32: spikes as 4-D {C, N, B, T}, box {32, 32, 1, 1}
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
  static constexpr int kKVTile = kAttnMaxN * kRowB;     // k or v rows of one step
  static constexpr int kDTile = HD * kRowB;             // D1 as fp16, HD rows
  // Ring slot: q tiles (2), k, v, D1 operand.
  static constexpr int kSlotBytes = 2 * kQTile + 2 * kKVTile + kDTile;
  static constexpr int kSlots = HD == 32 ? 4 : 2;
  static constexpr int kBarBytes = 256;
  // head_dim 32: one 2 KB spike staging tile per epilogue warp ([32 tokens]
  // [64 B], 64-byte swizzle) written out by TMA store.
  static constexpr int kStageOff = (kSlots * kSlotBytes + kBarBytes + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = HD == 32 ? 8 * 32 * kRowB : 0;
  static constexpr int kSmemBytes = kStageOff + kStageBytes + 1024;
  static constexpr int kCvtWarps = HD / 16;
  // TMEM: D1 buffers at columns 0 and HD (M = 64: HD columns each); D2
  // buffers at 2*HD and 4*HD (two M-tiles of HD columns each).
  static constexpr int kD2Col = 2 * HD;
  static constexpr int kTmemCols = HD == 32 ? 256 : 512;
  static_assert(6 * HD <= kTmemCols, "accumulators exceed the allocation");
};

// Byte offset of 16-byte chunk c of row r in a swizzled tile of kRowB rows.
template <int HD>
__device__ __forceinline__ int attn_swz(int r, int c) {
  if constexpr (HD == 32) return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
  else return r * 128 + ((c ^ (r & 7)) << 4);
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 1)
spikformer_attn_lif_kernel(const __grid_constant__ AttnParams p) {
  using Cfg = AttnCfg<HD>;
  constexpr int S = Cfg::kSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kSlotBytes);
  uint64_t* empty = full + S;
  uint64_t* dready = empty + S;
  uint64_t* d1_full = dready + S;        // [2]
  uint64_t* d1_empty = d1_full + 2;      // [2]
  uint64_t* d2_full = d1_empty + 2;      // [2]
  uint64_t* d2_empty = d2_full + 2;      // [2]
  uint64_t* drain = d2_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto slot_q = [&](int s, int m) { return smem + s * Cfg::kSlotBytes + m * Cfg::kQTile; };
  auto slot_k = [&](int s) { return smem + s * Cfg::kSlotBytes + 2 * Cfg::kQTile; };
  auto slot_v = [&](int s) { return slot_k(s) + Cfg::kKVTile; };
  auto slot_d = [&](int s) { return slot_v(s) + Cfg::kKVTile; };

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int N = p.N, C = p.C;
  const int n_mt = (N + 127) / 128;
  const int q_rows = min(N, 128);
  const int n_items = p.B * p.heads;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&dready[s], Cfg::kCvtWarps * 32);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&d1_full[j], 1);
      mbar_init(&d1_empty[j], Cfg::kCvtWarps * 32);
      mbar_init(&d2_full[j], 1);
      mbar_init(&d2_empty[j], kAttnEpiWarps * 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAttnTmaWarp && lane == 0) {
    prefetch_tmap(&p.tmap_q);
    prefetch_tmap(&p.tmap_k);
    prefetch_tmap(&p.tmap_v);
  }
  if (warp == kAttnMmaWarp) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();                            // q, k, v, state and out belong to the stream

  if (warp == kAttnTmaWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int bytes = 2 * p.kv_rows * Cfg::kRowB + n_mt * q_rows * Cfg::kRowB;
      int i = 0;
      bool stop = false;
      for (int it = blockIdx.x; it < n_items && !stop; it += gridDim.x) {
        const int b = it / p.heads, h = it % p.heads;
        for (int t = 0; t < p.T; ++t, ++i) {
          const int s = i % S;
          if (*abort_flag || !mbar_wait_bounded(&empty[s], ((i / S) & 1) ^ 1, p.timeout)) {
            if (!*abort_flag) atomicOr(p.err, kErrTimeoutEmpty);
            *abort_flag = 1; stop = true; break;
          }
          const int tb = t * p.B + b;
          mbar_arrive_expect_tx(&full[s], bytes);
          tma_load_3d(slot_k(s), &p.tmap_k, &full[s], h * HD, 0, tb);
          tma_load_3d(slot_v(s), &p.tmap_v, &full[s], h * HD, 0, tb);
          for (int m = 0; m < n_mt; ++m)
            tma_load_3d(slot_q(s, m), &p.tmap_q, &full[s], h * HD, m * 128, tb);
        }
      }
      // Let every load this thread issued land before the CTA can exit.
      for (int back = max(0, i - S); back < i; ++back)
        if (!mbar_wait_bounded(&full[back % S], (back / S) & 1, p.timeout))
          atomicOr(p.err, kErrTimeoutDrain);
    }
  } else if (warp == kAttnMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // GEMM 1: M = 64 (rows >= HD unused), N = HD, A and B MN-major.
      const uint32_t idesc1 = idesc_f16_major(64, HD, true, true);
      // GEMM 2: M = 128, N = HD, A K-major, B MN-major.
      const uint32_t idesc2 = idesc_f16_major(128, HD, false, true);
      constexpr uint32_t kKStep = (2 * Cfg::kSbo) >> 4;       // 16 rows along K, descriptor units
      bool stop = false;
      // GEMM 2 of step k: needs its D1 operand converted and a free D2 buffer.
      auto gemm2 = [&](int k) {
        const int s = k % S, j = k & 1;
        if (*abort_flag || !mbar_wait_bounded(&dready[s], (k / S) & 1, p.timeout) ||
            !mbar_wait_bounded(&d2_empty[j], ((k >> 1) & 1) ^ 1, p.timeout)) {
          if (!*abort_flag) atomicOr(p.err, kErrTimeoutAcc);
          *abort_flag = 1; stop = true; return;
        }
        tc_fence_after();
        const uint64_t b_desc = smem_desc_mnmajor(smem_u32(slot_d(s)), Cfg::kSbo, Cfg::kSbo,
                                                  Cfg::kLayout);
        for (int m = 0; m < n_mt; ++m) {
          const uint64_t a_desc = smem_desc_kmajor(smem_u32(slot_q(s, m)), Cfg::kSbo, Cfg::kLayout);
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks)   // A: +32 bytes along the row; B: +16 rows
            mma_f16(tmem + Cfg::kD2Col + j * 2 * HD + m * HD, a_desc + 2 * ks,
                    b_desc + ks * kKStep, idesc2, ks > 0 ? 1u : 0u);
        }
        mma_commit(&d2_full[j]);
        mma_commit(&empty[s]);           // the slot's tiles are read
      };
      int i = 0;
      for (int it = blockIdx.x; it < n_items && !stop; it += gridDim.x) {
        for (int t = 0; t < p.T && !stop; ++t, ++i) {
          const int s = i % S, j = i & 1;
          if (*abort_flag || !mbar_wait_bounded(&full[s], (i / S) & 1, p.timeout) ||
              !mbar_wait_bounded(&d1_empty[j], ((i >> 1) & 1) ^ 1, p.timeout)) {
            if (!*abort_flag) atomicOr(p.err, kErrTimeoutFull);
            *abort_flag = 1; stop = true; break;
          }
          tc_fence_after();
          // A: rows of HD channels; a 64-row M reads its second half one
          // 8-row group further (inside the tile; those D1 rows are unused).
          const uint64_t a_desc = smem_desc_mnmajor(smem_u32(slot_k(s)), Cfg::kSbo, Cfg::kSbo,
                                                    Cfg::kLayout);
          const uint64_t b_desc = smem_desc_mnmajor(smem_u32(slot_v(s)), Cfg::kSbo, Cfg::kSbo,
                                                    Cfg::kLayout);
          for (int ks = 0; ks < p.kv_rows / 16; ++ks)
            mma_f16(tmem + j * HD, a_desc + ks * kKStep, b_desc + ks * kKStep, idesc1,
                    ks > 0 ? 1u : 0u);
          mma_commit(&d1_full[j]);
          if (i > 0) gemm2(i - 1);
        }
      }
      if (!stop && i > 0) gemm2(i - 1);
      mma_commit(drain);
      if (!mbar_wait_bounded(drain, 0, p.timeout)) atomicOr(p.err, kErrTimeoutDrain);
    }
  } else if (warp >= kAttnCvtWarp0) {
    // ------------------------------------ D1 -> fp16 GEMM-2 operand (slot)
    // Row e (= channel) holds D1[e][0..HD).  An M = 64 accumulator keeps rows
    // 16q..16q+15 in lanes 32q..32q+15; warp 8+q reads lane quarter q.
    const int q = warp - kAttnCvtWarp0;
    if (q < Cfg::kCvtWarps) {
      const int e = 16 * q + lane;
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
      int i = 0;
      bool stop = false;
      for (int it = blockIdx.x; it < n_items && !stop; it += gridDim.x) {
        for (int t = 0; t < p.T; ++t, ++i) {
          const int s = i % S, j = i & 1;
          const bool ok = __all_sync(0xffffffffu, !*abort_flag &&
                                     mbar_wait_bounded(&d1_full[j], (i >> 1) & 1, p.timeout));
          if (!ok) {
            if (lane == 0 && !*abort_flag) atomicOr(p.err, kErrTimeoutAcc);
            *abort_flag = 1; stop = true; break;
          }
          tc_fence_after();
          float a[HD];
#pragma unroll
          for (int c0 = 0; c0 < HD; c0 += 32) {
            float a32[32];
            tmem_ld32(lane_base + j * HD + c0, a32);
#pragma unroll
            for (int u = 0; u < 32; ++u) a[c0 + u] = a32[u];
          }
          tc_fence_before();
          mbar_arrive(&d1_empty[j]);     // D1 buffer j may be overwritten
          if (lane < 16) {
#pragma unroll
            for (int c = 0; c < HD / 8; ++c) {
              uint32_t w[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const __half2 hv = __floats2half2_rn(a[8 * c + 2 * u], a[8 * c + 2 * u + 1]);
                w[u] = *reinterpret_cast<const uint32_t*>(&hv);
              }
              *reinterpret_cast<uint4*>(slot_d(s) + attn_swz<HD>(e, c)) =
                  make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
          fence_proxy_async_smem();      // generic-proxy writes -> tensor-core reads
          mbar_arrive(&dready[s]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    // GEMM-2 lane quarter warp%4 of M-tile warp/4.
    const int mt = warp >> 2;
    const int tok = mt * 128 + (warp & 3) * 32 + lane;
    uint8_t* stage = smem + Cfg::kStageOff + warp * 32 * Cfg::kRowB;   // head_dim 32 only
    int n_st = 0;
    const bool tok_ok = tok < N;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    int i = 0;
    bool stop = false;
    for (int it = blockIdx.x; it < n_items && !stop; it += gridDim.x) {
      const int b = it / p.heads, h = it % p.heads;
      const size_t state_row = (static_cast<size_t>(b) * N + tok) * C + h * HD;
      float vm[HD];
#pragma unroll
      for (int d = 0; d < HD; ++d)
        vm[d] = ((p.flags & kReadState) && tok_ok) ? p.state[state_row + d] : 0.f;
      for (int t = 0; t < p.T; ++t, ++i) {
        const int j = i & 1;
        // head_dim 32: the warp's staging tile must be read out by its
        // previous TMA store before it is rewritten.
        if (HD == 32 && n_st > 0) {
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
        }
        const bool ok = __all_sync(0xffffffffu, !*abort_flag &&
                                   mbar_wait_bounded(&d2_full[j], (i >> 1) & 1, p.timeout));
        if (!ok) {
          if (lane == 0 && !*abort_flag) atomicOr(p.err, kErrTimeoutAcc);
          *abort_flag = 1; stop = true; break;
        }
        tc_fence_after();
        // 32 channels at a time (bounded registers); the D2 buffer is
        // released once its last chunk is in registers.
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 32) {
          float x[32];
          if (mt < n_mt) tmem_ld32(lane_base + Cfg::kD2Col + j * 2 * HD + mt * HD + c0, x);
          if (c0 + 32 == HD) {
            tc_fence_before();
            mbar_arrive(&d2_empty[j]);   // D2 buffer j may be overwritten
          }
          if (mt < n_mt) {
            uint32_t packed[16];
#pragma unroll
            for (int d = 0; d < 32; d += 2) {
              bool sp[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const float xs = x[d + u] * p.scale;   // exact: a multiple of scale
                float& v = vm[c0 + d + u];
                float hv;
                if (p.lif_half) hv = fmaf(v, 0.5f, xs * 0.5f);
                else hv = __fadd_rn(__fmul_rn(v, p.decay), __fdiv_rn(xs, p.tau));
                sp[u] = hv >= p.v_th;
                v = sp[u] ? p.v_reset : hv;
              }
              packed[d / 2] = (sp[0] ? 0x3C00u : 0u) | (sp[1] ? 0x3C000000u : 0u);
            }
            if constexpr (HD == 32) {
              // Row `lane` of the staging tile; tokens past N are not stored.
#pragma unroll
              for (int c = 0; c < 4; ++c)
                *reinterpret_cast<uint4*>(stage + attn_swz<32>(lane, c)) =
                    make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_4d(&p.tmap_out, stage, h * HD + c0, mt * 128 + (warp & 3) * 32, b, t);
                bulk_commit_group();
              }
              ++n_st;
            } else if (tok_ok) {
              uint4* o = reinterpret_cast<uint4*>(
                  p.out + (static_cast<size_t>(t * p.B + b) * N + tok) * C + h * HD + c0);
#pragma unroll
              for (int c = 0; c < 4; ++c)
                o[c] = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
            }
          }
        }
      }
      if (!stop && (p.flags & kWriteState) && tok_ok) {
#pragma unroll
        for (int d = 0; d < HD; ++d) p.state[state_row + d] = vm[d];
      }
    }
    if (HD == 32 && n_st > 0 && lane == 0) bulk_wait_group<0>();   // stores complete before exit
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAttnMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace snn
