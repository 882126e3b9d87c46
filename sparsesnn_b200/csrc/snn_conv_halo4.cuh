// Four-timestep halo variant of the fused 2:4-sparse conv for stride-1 3x3
// "same" convolutions with at most 64 output channels and a spiking
// epilogue (SEW-ResNet stage 1 on CIFAR: 64 -> 64 channels at 32 x 32).
//
// Why: an implicit-GEMM MMA whose A and B operands both move from one MMA to
// the next costs about 120-150 cycles whatever N <= 128, while an N = 256
// MMA runs at its operand rate (about 144 cycles at M = 64).  So each MMA
// here covers 8 x 8 output pixels x 4 timesteps (N = 256) instead of 128
// pixels of one timestep: half the MMAs for the same work.
//
// How: the input halo of a tile (10 x 10 pixels) is loaded for four
// timesteps by ONE TMA box from a tensor map whose dimensions are ordered
// (C, W, T, H, B), so shared memory holds [halo row][timestep][halo column]
// 128-byte pixel rows.  The 8-pixel groups of a tap's B operand are then
// uniformly spaced (one timestep block of 10 pixels apart): group g is halo
// row kh + g/4 of timestep g%4, columns kw..kw+7.  Accumulator column
// n = 32*r + 8*t + c holds output row r, timestep t, column c.
//
// TMEM: the 256-column accumulator is single-buffered (the 2:4 metadata
// takes columns from 256 on); the epilogue copies its columns to registers
// and releases the accumulator before running the neurons, so the next
// tile's MMAs wait only for that copy.
//
// Warp roles (12 warps): 0..7 epilogue (TMEM lane quarter q = warp % 4,
// tile half h = warp / 4: output rows 4h..4h+3); 8..11 load the metadata,
// then warp 10 issues MMAs and owns TMEM and warp 11 drives TMA.  An
// epilogue thread owns channel 16q + lane%16 of two output rows
// (4h + 2*(lane/16) and the next), i.e. 16 pixels over all timesteps, whose
// membranes stay in registers.  A warp ballot per (timestep, pixel pair)
// gathers 2 x 16 channels' spikes; each lane keeps the ballots of one pixel
// column and expands them into 16-byte fp16 chunks of a staging tile that
// one TMA store writes out (with the SEW residual, loaded into the tile by
// TMA, added in place).
#pragma once
#include "snn_conv_halo.cuh"

namespace snn {

constexpr int kH4Threads = 384;
constexpr int kH4MmaWarp = 10;
constexpr int kH4TmaWarp = 11;
constexpr int kH4MaxStages = 4;
constexpr int kH4Ts = 4;                          // timesteps per MMA
constexpr int kH4MetaCol = 256;                   // after the 256 accumulator columns
constexpr int kH4TmemCols = 512;
// One output staging tile: [4 t][8 rows][8 columns] x 64 channels fp16,
// 128-byte pixel rows with the 128-byte TMA swizzle.
constexpr int kH4OutBytes = kH4Ts * 64 * 128;
constexpr int kH4StoreBar = 1;                    // named barrier of the 8 epilogue warps

// Like tmem_ld16x2_32, with the second 16-thread half reading 64 columns on.
__device__ __forceinline__ void tmem_ld16x2_32_split64(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], 64;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <int MODE, bool RES>
__global__ void __launch_bounds__(kH4Threads, 1)
fused_sparse_conv_halo4_kernel(const __grid_constant__ HaloParams hp) {
  static_assert(MODE != kModeNone, "spiking epilogues or the fp16 BN output");
  constexpr int KS = 3;
  const ConvParams& p = hp.c;
  constexpr int kAKb = 64 * (kKB / 2) * 2;       // resident weight bytes per k-block (64 rows)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                                              // resident weights
  uint8_t* sH = smem + hp.a_bytes;                                 // halo stages
  uint8_t* sO = sH + hp.halo_stages * hp.halo_stride;              // 2 output staging tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(sO + 2 * kH4OutBytes);
  uint64_t* empty = full + kH4MaxStages;
  uint64_t* a_full = empty + kH4MaxStages;
  uint64_t* acc_full = a_full + 1;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* meta_ready = acc_empty + 1;
  uint64_t* drain = meta_ready + 1;
  uint64_t* res_full = drain + 1;           // [2]: residual box landed in a staging tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int first_pt = blockIdx.x;
  const int pt_step = gridDim.x;
  const int n_meta = 2 * p.n_kb;
  const int n_pass = (p.T + kH4Ts - 1) / kH4Ts;
  const int S = hp.halo_stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(a_full, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kEpiThreads);
    mbar_init(meta_ready, 128);
    mbar_init(drain, 1);
    mbar_init(&res_full[0], 1);
    mbar_init(&res_full[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kH4TmaWarp && lane == 0) {
    prefetch_tmap(&p.tmap_a); prefetch_tmap(&p.tmap_b[0]); prefetch_tmap(&p.tmap_b[1]);
    if (RES) prefetch_tmap(&p.tmap_b[2]);
  }
  if (warp == kH4MmaWarp) { tmem_alloc(tmem_slot, kH4TmemCols); tmem_relinquish(); }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kH4TmaWarp && lane == 0) {
    // The resident weights: one 3-D box ([k-block][64 rows][32 elements]).
    mbar_arrive_expect_tx(a_full, hp.a_bytes);
    tma_load_3d(sA, &p.tmap_a, a_full, 0, 0, 0);
  }
  if (warp >= kEpiWarps) {
    // ------------------------------------------- metadata into TMEM (warps 8..11)
    // M = 64 takes rows 16q..16q+15 from lanes 32q..32q+15; the other lanes
    // get the dense pattern.
    const int q = warp & 3;
    const int row = lane < 16 ? q * 16 + lane : -1;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t* src = p.meta + max(row, 0);
    constexpr int kChunk = 40;
    for (int j = 0; j < n_meta; j += kChunk) {
      uint32_t r[kChunk];
#pragma unroll
      for (int i = 0; i < kChunk; ++i)
        r[i] = (j + i < n_meta && row >= 0) ? __ldg(src + static_cast<size_t>(j + i) * kBM)
                                            : 0x44444444u;
#pragma unroll
      for (int u = 0; u < kChunk / 8; ++u) {
        if (j + 8 * u < n_meta) {
          uint32_t r8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) r8[i] = r[8 * u + i];
          tmem_st8(lane_base + kH4MetaCol + j + 8 * u, r8);
        }
      }
    }
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive(meta_ready);
  }

  if (warp == kH4TmaWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      pdl_wait();                        // activations come from the previous kernel
      int stage = 0; uint32_t phase = 0;
      int issued = 0;
      bool stop = false;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        const TileCoord tc = tile_coord(p, pt);
        for (int ps = 0; ps < n_pass && !stop; ++ps) {
          for (int cb = 0; cb < p.cin_blocks; ++cb) {
            if (*abort_flag) { stop = true; break; }
            if (!mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutEmpty); *abort_flag = 1; stop = true; break;
            }
            mbar_arrive_expect_tx(&full[stage], hp.halo_bytes);
            // Coordinates (channel, column, timestep, row, image); timesteps
            // past T and pixels outside the image read as zero.
            tma_load_5d(sH + stage * hp.halo_stride, &p.tmap_b[0], &full[stage], cb * kKB,
                        tc.w0 - p.pad, ps * kH4Ts, tc.h0 - p.pad, tc.n0);
            ++issued;
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
        }
      }
      const int n_wait = min(issued, S);
      for (int i = 0; i < n_wait; ++i) {
        const int back = issued - 1 - i;
        if (!mbar_wait_bounded(&full[back % S], (back / S) & 1, p.timeout_ns))
          atomicOr(p.err, kErrTimeoutFull);
      }
      if (!mbar_wait_bounded(a_full, 0, p.timeout_ns)) atomicOr(p.err, kErrTimeoutFull);
    }
  } else if (warp == kH4MmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(64, 8 * 8 * kH4Ts, true);
      bool ok = mbar_wait_bounded(meta_ready, 0, p.timeout_ns);
      ok = ok && mbar_wait_bounded(a_full, 0, p.timeout_ns);
      if (!ok) { atomicOr(p.err, kErrTimeoutMeta); *abort_flag = 1; }
      tc_fence_after();
      // 8-pixel groups one timestep block (halo_w pixel rows) apart.
      const uint32_t sbo = static_cast<uint32_t>(hp.halo_w) * 128;
      const uint64_t a_desc0 = smem_desc_kmajor(smem_u32(sA), 512, 4);
      const uint64_t h_desc0 = smem_desc_kmajor(smem_u32(sH), sbo, 2);
      const int halo_row16 = kH4Ts * hp.halo_w * 8;    // one halo row, all timesteps, 16-byte units
      int stage = 0; uint32_t phase = 0;
      int it = 0;
      bool stop = *abort_flag != 0;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        for (int ps = 0; ps < n_pass && !stop; ++ps) {
          if (!mbar_wait_bounded(acc_empty, (it & 1) ^ 1, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutAccEmpty); *abort_flag = 1; stop = true; break;
          }
          tc_fence_after();
          for (int cb = 0; cb < p.cin_blocks; ++cb) {
            if (!mbar_wait_bounded(&full[stage], phase, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutFull); *abort_flag = 1; stop = true; break;
            }
            tc_fence_after();
            const uint64_t hd = h_desc0 + static_cast<uint32_t>(stage * hp.halo_stride >> 4);
#pragma unroll
            for (int kh = 0; kh < KS; ++kh) {
#pragma unroll
              for (int kw = 0; kw < KS; ++kw) {
                const int kb = (kh * KS + kw) * p.cin_blocks + cb;
                const uint64_t ad = a_desc0 + static_cast<uint32_t>(kb * (kAKb >> 4));
                const uint64_t bd = hd + static_cast<uint32_t>(kh * halo_row16 + kw * 8);
                const uint32_t e_addr = tmem + kH4MetaCol + 2 * kb;
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                  const bool first = (cb == 0 && kh == 0 && kw == 0 && s == 0);
                  mma_sp_f16(tmem, ad + 2 * s, bd + 4 * s, e_addr, idesc | static_cast<uint32_t>(s),
                             first ? 0u : 1u);
                }
              }
            }
            mma_commit(&empty[stage]);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
          if (stop) break;
          mma_commit(acc_full);
          ++it;
        }
      }
      mma_commit(drain);
      if (!mbar_wait_bounded(drain, 0, p.timeout_ns)) atomicOr(p.err, kErrTimeoutDrain);
    }
  } else if (warp < kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = warp >> 2;
    const int ch = q * 16 + (lane & 15);         // neuron phase: this thread's channel
    const bool cvalid = ch < p.F;
    const float sc = cvalid ? p.scale[ch] : 0.f;
    const float bi = cvalid ? p.bias[ch] : 0.f;
    const float sx = MODE == kModeLifHalf ? sc * 0.5f : sc;
    const float bx = MODE == kModeLifHalf ? bi * 0.5f : bi;
    const uint32_t acc_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + half * 128;
    const int r0 = half * 4 + (lane >> 4) * 2;   // neuron phase: tile rows r0, r0 + 1
    // Staging phase: lane l writes channels 16q + 8*(l%2) .. +7 (one 16-byte
    // chunk) of tile pixel (4*half + 2*sel + l/16, (l/2) % 8), sel = 0, 1,
    // for each of the pass's timesteps.
    const int sub = lane & 1;
    const int scol = (lane >> 1) & 7, srow_in = lane >> 4;
    pdl_wait();                                  // residual, output and state

    // Output path: each pass's spikes (plus the SEW residual) are assembled
    // in a staging tile laid out as the TMA box {64 ch, 8 w, 8 h, 1, 4 t} and
    // leave through one TMA store issued by thread 0; out-of-range pixels,
    // channels and timesteps of the box are not written.  Global stores from
    // the epilogue warps would share the SM's load/store path with the MMAs'
    // shared-memory operand reads and slow them down.  The SEW residual
    // arrives by TMA into the staging tile the pass will use; the two tiles
    // alternate, and thread 0 waits for a tile's previous store to finish
    // reading it before the residual load or the next writes reuse it.
    const bool storer = warp == 0 && lane == 0;
    auto issue_res = [&](int pt_n, int ps_n, int buf) {   // residual of pass (pt_n, ps_n)
      const TileCoord tn = tile_coord(p, pt_n);
      mbar_arrive_expect_tx(&res_full[buf], kH4OutBytes);
      tma_load_5d(sO + buf * kH4OutBytes, &p.tmap_b[2], &res_full[buf], 0, tn.w0, tn.h0, tn.n0,
                  ps_n * kH4Ts);
    };
    if (RES && storer && first_pt < p.n_px_tiles) issue_res(first_pt, 0, 0);

    int it = 0;
    bool stop = false;
    for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
      const TileCoord tc = tile_coord(p, pt);
      auto px_of = [&](int r, int c) -> int {    // tile row/column -> output pixel (-1: outside)
        const int oh = tc.h0 + r, ow = tc.w0 + c;
        return (oh < p.OH && ow < p.OW) ? (tc.n0 * p.OH + oh) * p.OW + ow : -1;
      };
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int px = px_of(r0 + (i >> 3), i & 7);
        v[i] = ((p.flags & kReadState) && cvalid && px >= 0)
                   ? p.state[static_cast<size_t>(px) * p.F + ch] : 0.f;
      }
      for (int ps = 0; ps < n_pass; ++ps) {
        const int t0 = ps * kH4Ts;
        const int buf = it & 1;
        bool fail = !mbar_wait_bounded(acc_full, it & 1, p.timeout_ns);
        fail = __any_sync(0xffffffffu, fail || *abort_flag);
        // A failed wait skips the work but still reaches the pass's barrier,
        // where the eight warps agree to stop.
        if (!fail) {
        tc_fence_after();
        float acc0[32], acc1[32];                // rows r0 and r0 + 1: [t*8 + column]
        tmem_ld16x2_32_split64(acc_base, acc0);
        tmem_ld16x2_32_split64(acc_base + 32, acc1);
        tc_fence_before();
        mbar_arrive(acc_empty);                  // accumulator copied: the next MMAs may start
        // Neurons; each step's spikes of the warp are gathered by a ballot
        // (bits 0..15: channels 16q.. of the lower lanes' pixel, 16..31: of
        // the upper lanes' pixel two rows down), and lane l keeps the ballots
        // of the pixel column it writes.
        if constexpr (MODE == kModeBnF16) {
          // No neuron: each thread writes its channel's bn (+ residual, added
          // in fp32 and rounded once) straight into the staging tile, at
          // pixel (t, row, column) = byte ((t*8 + row)*8 + column)*128 +
          // (16-byte chunk ch/8 XOR column)*16 + (ch%8)*2.
          if constexpr (RES) {
            if (!mbar_wait_bounded(&res_full[buf], (it >> 1) & 1, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutRes); fail = true;
            }
          }
          uint8_t* tile = sO + buf * kH4OutBytes;
#pragma unroll
          for (int t = 0; t < kH4Ts; ++t) {
#pragma unroll
            for (int a = 0; a < 2; ++a) {
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                float x = fmaf(a ? acc1[t * 8 + c] : acc0[t * 8 + c], sc, bi);
                const int prow = (t * 8 + r0 + a) * 8 + c;
                __half* dst = reinterpret_cast<__half*>(tile + prow * 128 + ((((ch >> 3) ^ c)) << 4)) +
                              (ch & 7);
                if constexpr (RES) x = __fadd_rn(x, fail ? 0.f : __half2float(*dst));
                if (cvalid && !fail) *dst = __float2half_rn(x);
              }
            }
          }
          fence_proxy_async_smem();
        } else {
        uint32_t pk[2][kH4Ts];
#pragma unroll
        for (int t = 0; t < kH4Ts; ++t) {
          pk[0][t] = 0u; pk[1][t] = 0u;
#pragma unroll
          for (int a = 0; a < 2; ++a) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const float x = fmaf(a ? acc1[t * 8 + c] : acc0[t * 8 + c], sx, bx);
              // Timesteps past T (zero input) must not advance the membrane.
              const bool spike = t0 + t < p.T &&
                                 neuron_step<MODE>(v[a * 8 + c], x, p.decay, p.tau, p.v_th, p.v_reset);
              const uint32_t m = __ballot_sync(0xffffffffu, spike);
              if (((lane >> 1) & 7) == c) pk[a][t] = m;
            }
          }
        }
        if constexpr (RES) {
          if (!mbar_wait_bounded(&res_full[buf], (it >> 1) & 1, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutRes); fail = true;
          }
        }
        // pk[a][t] holds, for this lane's column, rows 4h + a (bits 0..15) and
        // 4h + 2 + a (bits 16..31); the lane writes row 4h + 2*sel + l/16,
        // 16-byte chunk 2q + l%2 (swizzled by the pixel row's index mod 8,
        // which is the column).
        uint8_t* tile = sO + buf * kH4OutBytes;
#pragma unroll
        for (int u = 0; u < 2 * kH4Ts; ++u) {
          const int t = u >> 1, sel = u & 1;
          const uint32_t m = srow_in ? pk[1][t] : pk[0][t];
          const uint32_t bits = (m >> (16 * sel + 8 * sub)) & 0xffu;
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            w[k] = ((bits >> (2 * k)) & 1u ? 0x3C00u : 0u) | ((bits >> (2 * k + 1)) & 1u ? 0x3C000000u : 0u);
          uint4 o = make_uint4(w[0], w[1], w[2], w[3]);
          const int prow = (t * 8 + half * 4 + 2 * sel + srow_in) * 8 + scol;
          uint4* dst = reinterpret_cast<uint4*>(tile + prow * 128 + (((2 * q + sub) ^ scol) << 4));
          if constexpr (RES) {
            const uint4 r = fail ? make_uint4(0, 0, 0, 0) : *dst;
            __half2* hp2 = reinterpret_cast<__half2*>(&o);
            const __half2* rb = reinterpret_cast<const __half2*>(&r);
#pragma unroll
            for (int k = 0; k < 4; ++k) hp2[k] = __hadd2(hp2[k], rb[k]);
          }
          if (!fail) *dst = o;
        }
        fence_proxy_async_smem();
        }
        }
        // Thread 0 first waits until the other tile's previous store has read
        // it, so after this barrier that tile is free for the next pass.
        if (storer) bulk_wait_group_read<0>();
        if (named_barrier_or(kH4StoreBar, kEpiThreads, fail)) {
          atomicOr(p.err, kErrTimeoutAcc); stop = true; break;
        }
        if (storer) {
          tma_store_5d(&p.tmap_b[1], sO + buf * kH4OutBytes, 0, tc.w0, tc.h0, tc.n0, t0);
          bulk_commit_group();
          if constexpr (RES) {
            // The next pass's residual into the other tile.
            int pt_n = pt, ps_n = ps + 1;
            if (ps_n == n_pass) { pt_n += pt_step; ps_n = 0; }
            if (pt_n < p.n_px_tiles) issue_res(pt_n, ps_n, buf ^ 1);
          }
        }
        ++it;
      }
      if (!stop && (p.flags & kWriteState)) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int px = px_of(r0 + (i >> 3), i & 7);
          if (cvalid && px >= 0) p.state[static_cast<size_t>(px) * p.F + ch] = v[i];
        }
      }
    }
    if (storer) bulk_wait_group<0>();            // stores complete before the CTA exits
    if (stop) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kH4MmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kH4TmemCols);
  }
}

}  // namespace snn
