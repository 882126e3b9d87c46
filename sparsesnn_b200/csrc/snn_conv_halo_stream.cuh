// Streaming-weight halo variant for stride-1 3x3 convolutions whose weight
// slice is too large to stay resident (e.g. Cin = 256), on images of at
// least 8x8.  A tile is 8x8 output pixels of one image for all T timesteps
// (T <= 4): ONE MMA per tap covers them all (UMMA N = 64*T), so every weight
// tile that enters shared memory is read once per tap for all timesteps.
//
// Per (tile, 64-channel slice cb): the producer loads the T input halos
// (10x10 pixels each) as ONE 5D TMA box from a (C, W, T, H, B) view of the
// activations, so shared memory holds [halo row][timestep][halo column]
// 128-byte pixel rows; a tap's B operand starts at row (kh*T*10 + kw) and
// its 8-pixel groups are one timestep block (10 rows) apart: group g is
// output row g/T of timestep g%T, and accumulator column 8*(T*r + t) + c
// holds output row r, timestep t, column c.  The slice's weights arrive in
// three kernel-row stages, each ONE 3D box of 3 taps x 128 rows.  A TMA box
// costs a fixed few hundred cycles whatever its size, so the kernel issues
// as few, large boxes as it can.
//
// SMALL (4x4 images, e.g. ResNet stage 4 on CIFAR): a tile is 4 whole images.
// Rows of 4 pixels cannot form the 8-pixel groups of one halo row, so per
// slice the producer loads three column-shifted boxes (kw = 0, 1, 2) from a
// (C, W, T, B, H) view: [halo row][image][timestep][4 columns], 6 x 4 x T x 4
// pixel rows.  Tap (kh, kw) then reads 16*T*4 CONSECUTIVE rows of box kw
// starting at halo row kh (a plain K-major operand, groups 1024 bytes
// apart); accumulator column ((r*4 + image)*T + t)*4 + c.  Weights come per
// kw as one 4-D box of the three taps (0..2, kw).
//
// Warp roles: 0..7 epilogue, 8..11 metadata, then 10 = MMA + TMEM owner,
// 11 = halo loads, 8 and 9 = weight loads.
#pragma once
#include "snn_conv_halo.cuh"

namespace snn {

constexpr int kHsMaxT = 4;
constexpr int kHsBN = 64;
constexpr int kHsHaloStages = 2;                   // each stage: the halos of all T timesteps
constexpr int kHsAStages = 4;
constexpr int kHsAStageBytes = 3 * kABytes;        // one kernel row: 3 taps, one 3D TMA box
constexpr int kHsHaloBytes = 10 * 10 * kKB * 2;    // 12800 per timestep
constexpr int kHsHaloStride = kHsMaxT * kHsHaloBytes;  // 51200 (1024-aligned)
constexpr int kHsSmallBytes = 6 * 4 * 4 * kKB * 2;     // SMALL: one kw box per timestep (12288)
constexpr int kHsMetaCol = 256;
constexpr int kHsSmemBytes = kHsAStages * kHsAStageBytes + kHsHaloStages * kHsHaloStride +
                             kEpiWarps * kXposeBytes + 512 + 1024;

template <int MODE, bool RES, bool SMALL = false>
__global__ void __launch_bounds__(kHaloThreads, 1)
fused_sparse_conv_halo_stream_kernel(const __grid_constant__ ConvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                                              // weight ring
  uint8_t* sH = smem + kHsAStages * kHsAStageBytes;                // halo ring
  uint8_t* sX = sH + kHsHaloStages * kHsHaloStride;                // epilogue transposes
  uint64_t* a_full = reinterpret_cast<uint64_t*>(sX + kEpiWarps * kXposeBytes);
  uint64_t* a_empty = a_full + kHsAStages;
  uint64_t* h_full = a_empty + kHsAStages;
  uint64_t* h_empty = h_full + kHsHaloStages;
  uint64_t* acc_full = h_empty + kHsHaloStages;   // [kHsMaxT]
  uint64_t* acc_empty = acc_full + kHsMaxT;       // [kHsMaxT]
  uint64_t* meta_ready = acc_empty + kHsMaxT;
  uint64_t* drain = meta_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int m_tile = blockIdx.x % p.n_m;
  const int first_pt = blockIdx.x / p.n_m;
  const int pt_step = gridDim.x / p.n_m;
  const int n_meta = 2 * p.n_kb;
  const int T = p.T;
  // CTAs start their channel-slice loop at different slices so that the CTAs
  // sharing a weight slice do not all request the same weight rows at once.
  const int cb_rot = first_pt % p.cin_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kHsAStages; ++s) { mbar_init(&a_full[s], 1); mbar_init(&a_empty[s], 1); }
    for (int s = 0; s < kHsHaloStages; ++s) { mbar_init(&h_full[s], 1); mbar_init(&h_empty[s], 1); }
    for (int t = 0; t < kHsMaxT; ++t) { mbar_init(&acc_full[t], 1); mbar_init(&acc_empty[t], kEpiThreads); }
    mbar_init(meta_ready, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kHaloTmaWarp && lane == 0) { prefetch_tmap(&p.tmap_b[0]); prefetch_tmap(&p.tmap_b[1]); }
  if (warp == kHaloMmaWarp) { tmem_alloc(tmem_slot, kHaloTmemCols); tmem_relinquish(); }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= kEpiWarps) {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t* src = p.meta + (static_cast<size_t>(m_tile) * n_meta) * kBM + row;
    // Up to 40 columns' loads in flight per lane (a 512-channel 3x3 layer has
    // 144 metadata columns: four round trips instead of eighteen).
    constexpr int kChunk = 40;
    for (int j = 0; j < n_meta; j += kChunk) {
      uint32_t r[kChunk];
#pragma unroll
      for (int i = 0; i < kChunk; ++i)
        r[i] = (j + i < n_meta) ? __ldg(src + static_cast<size_t>(j + i) * kBM) : 0x44444444u;
#pragma unroll
      for (int u = 0; u < kChunk / 8; ++u) {
        if (j + 8 * u < n_meta) {
          uint32_t r8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) r8[i] = r[8 * u + i];
          tmem_st8(lane_base + kHsMetaCol + j + 8 * u, r8);
        }
      }
    }
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive(meta_ready);
  }

  if (warp == kHaloTmaWarp || warp == 8 || warp == 9) {
    // ----------------------------------------------------------- producers
    // Warp 11 loads the halos; warps 8 and 9 load the weight stages (fill j
    // by warp 8 + j % 2).  A thread issues tensor copies one after another,
    // so spreading them over three warps keeps more boxes in flight.
    if (lane == 0) {
      const bool halo_warp = warp == kHaloTmaWarp;
      if (halo_warp) pdl_wait();         // activations come from the previous kernel
      const int wprod = warp - 8;
      int as = 0, hs = 0; uint32_t aph = 0, hph = 0;
      int a_seq = 0, a_issued = 0, a_last = -1, h_issued = 0;
      bool stop = false;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        const TileCoord tc = tile_coord(p, pt);
        for (int cbi = 0; cbi < p.cin_blocks && !stop; ++cbi) {
          const int cb = (cbi + cb_rot) % p.cin_blocks;
          if (*abort_flag) { stop = true; break; }
          if (halo_warp) {
            for (int u = 0; u < (SMALL ? 3 : 1) && !stop; ++u) {
              if (!mbar_wait_bounded(&h_empty[hs], hph ^ 1, p.timeout_ns)) {
                atomicOr(p.err, kErrTimeoutEmpty); *abort_flag = 1; stop = true; break;
              }
              if constexpr (SMALL) {
                // Box kw = u: coordinates (channel, column, timestep, image, row).
                mbar_arrive_expect_tx(&h_full[hs], T * kHsSmallBytes);
                tma_load_5d(sH + hs * kHsHaloStride, &p.tmap_b[0], &h_full[hs], cb * kKB, u - 1, 0,
                            tc.n0, -1);
              } else {
                // All T halos in one box: coordinates (channel, column,
                // timestep, row, image).
                mbar_arrive_expect_tx(&h_full[hs], T * kHsHaloBytes);
                tma_load_5d(sH + hs * kHsHaloStride, &p.tmap_b[0], &h_full[hs], cb * kKB,
                            tc.w0 - 1, 0, tc.h0 - 1, tc.n0);
              }
              ++h_issued;
              if (++hs == kHsHaloStages) { hs = 0; hph ^= 1; }
            }
            continue;
          }
          for (int kh = 0; kh < 3 && !stop; ++kh, ++a_seq) {
            if ((a_seq & 1) == wprod) {
              if (*abort_flag) { stop = true; break; }
              if (!mbar_wait_bounded(&a_empty[as], aph ^ 1, p.timeout_ns)) {
                atomicOr(p.err, kErrTimeoutEmpty); *abort_flag = 1; stop = true; break;
              }
              mbar_arrive_expect_tx(&a_full[as], kHsAStageBytes);
              if constexpr (SMALL) {
                // Weights of taps (0..2, kw = kh loop index): [kh][128 rows][32 el].
                tma_load_4d(sA + as * kHsAStageBytes, &p.tmap_b[1], &a_full[as], cb * (kKB / 2),
                            m_tile * kBM, 0, kh);
              } else {
                // Weights of taps (kh, 0..2) for slice cb: [tap][128 rows][32 el].
                tma_load_3d(sA + as * kHsAStageBytes, &p.tmap_b[1], &a_full[as], cb * (kKB / 2),
                            m_tile * kBM, kh * 3);
              }
              ++a_issued; a_last = a_seq;
            }
            if (++as == kHsAStages) { as = 0; aph ^= 1; }
          }
        }
      }
      // Let every load this warp issued land before the CTA can exit.
      for (int i = 0; i < min(h_issued, kHsHaloStages); ++i) {
        const int back = h_issued - 1 - i;
        if (!mbar_wait_bounded(&h_full[back % kHsHaloStages], (back / kHsHaloStages) & 1, p.timeout_ns))
          atomicOr(p.err, kErrTimeoutFull);
      }
      for (int i = 0; i < min(a_issued, kHsAStages / 2); ++i) {
        const int back = a_last - 2 * i;
        if (!mbar_wait_bounded(&a_full[back % kHsAStages], (back / kHsAStages) & 1, p.timeout_ns))
          atomicOr(p.err, kErrTimeoutFull);
      }
    }
  } else if (warp == kHaloMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, kHsBN * T, true);
      if (!mbar_wait_bounded(meta_ready, 0, p.timeout_ns)) { atomicOr(p.err, kErrTimeoutMeta); *abort_flag = 1; }
      tc_fence_after();
      const uint32_t a_base = smem_u32(sA);
      const uint32_t h_base = smem_u32(sH);
      int as = 0, hs = 0; uint32_t aph = 0, hph = 0;
      int tile_it = 0;
      bool stop = *abort_flag != 0;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        // Every timestep's accumulator must be drained by the epilogue.
        for (int t = 0; t < T && !stop; ++t) {
          if (!mbar_wait_bounded(&acc_empty[t], (tile_it & 1) ^ 1, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutAccEmpty); *abort_flag = 1; stop = true;
          }
        }
        if (stop) break;
        tc_fence_after();
        for (int cbi = 0; cbi < p.cin_blocks && !stop; ++cbi) {
          const int cb = (cbi + cb_rot) % p.cin_blocks;
          if constexpr (!SMALL) {
            if (!mbar_wait_bounded(&h_full[hs], hph, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutFull); *abort_flag = 1; stop = true; break;
            }
          }
          tc_fence_after();
          for (int kh = 0; kh < 3; ++kh) {      // SMALL: this index is kw
            if constexpr (SMALL) {
              if (!mbar_wait_bounded(&h_full[hs], hph, p.timeout_ns)) {
                atomicOr(p.err, kErrTimeoutFull); *abort_flag = 1; stop = true; break;
              }
            }
            const uint32_t hstage = h_base + hs * kHsHaloStride;
            if (!mbar_wait_bounded(&a_full[as], aph, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutFull); *abort_flag = 1; stop = true; break;
            }
            tc_fence_after();
            const uint32_t abase = a_base + as * kHsAStageBytes;
            if constexpr (SMALL) {
              const int kw = kh;
#pragma unroll
              for (int r = 0; r < 3; ++r) {     // kernel row
                const int kb = (r * 3 + kw) * p.cin_blocks + cb;
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                  const uint32_t ecol = kHsMetaCol + 2 * kb + s;
                  const uint32_t acc = (cbi > 0 || kw > 0 || r > 0 || s > 0) ? 1u : 0u;
                  const uint64_t adesc = smem_desc_kmajor(abase + r * kABytes + 32 * s, 512, 4);
                  const uint64_t bdesc = smem_desc_kmajor(hstage + r * (16 * T * 128) + 64 * s, 1024, 2);
                  mma_sp_f16(tmem, adesc, bdesc, tmem + (ecol & ~1u), idesc | (ecol & 1u), acc);
                }
              }
              mma_commit(&h_empty[hs]);        // this kw box is consumed
              if (++hs == kHsHaloStages) { hs = 0; hph ^= 1; }
            } else {
#pragma unroll
              for (int kw = 0; kw < 3; ++kw) {
                const int kb = (kh * 3 + kw) * p.cin_blocks + cb;
                const uint32_t boff = static_cast<uint32_t>(kh * T * 10 + kw) * 128;
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                  const uint32_t ecol = kHsMetaCol + 2 * kb + s;
                  const uint32_t e_addr = tmem + (ecol & ~1u);
                  const uint32_t id = idesc | (ecol & 1u);
                  const uint64_t adesc = smem_desc_kmajor(abase + kw * kABytes + 32 * s, 512, 4);
                  const uint32_t acc = (cbi > 0 || kh > 0 || kw > 0 || s > 0) ? 1u : 0u;
                  mma_sp_f16(tmem, adesc, smem_desc_kmajor(hstage + boff + 64 * s, 1280, 2), e_addr, id,
                             acc);
                }
              }
            }
            mma_commit(&a_empty[as]);
            if (++as == kHsAStages) { as = 0; aph ^= 1; }
          }
          if (stop) break;
          if constexpr (!SMALL) {
            mma_commit(&h_empty[hs]);        // this slice's halos are consumed
            if (++hs == kHsHaloStages) { hs = 0; hph ^= 1; }
          }
        }
        if (stop) break;
        for (int t = 0; t < T; ++t) mma_commit(&acc_full[t]);
        ++tile_it;
      }
      mma_commit(drain);
      if (!mbar_wait_bounded(drain, 0, p.timeout_ns)) atomicOr(p.err, kErrTimeoutDrain);
    }
  } else if (warp < kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = warp >> 2;                  // pixel columns [32*half, 32*half+32)
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int cout = m_tile * kBM + row;
    const bool cvalid = cout < p.F;
    const int cbase = m_tile * kBM + q * 32;
    const bool warp_live = cbase < p.F;
    const float sc = cvalid ? p.scale[cout] : 0.f;
    const float bi = cvalid ? p.bias[cout] : 0.f;
    const float sx = MODE == kModeLifHalf ? sc * 0.5f : sc;
    const float bx = MODE == kModeLifHalf ? bi * 0.5f : bi;
    const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
    const int nchunk8 = max(0, min(4, (p.F - cbase) / 8));
    const bool chunk_ok = (lane & 3) < nchunk8;
    uint8_t* xb = sX + warp * kXposeBytes;
    // With p.tma_out the transpose tile ({32 ch, 8 w, 4 h} in the 64-byte
    // TMA swizzle) leaves by a TMA store issued by lane 0, which waits for it
    // to read the tile before the tile is rewritten.
    const bool tma_out = p.tma_out != 0;
    int n_st = 0;
    pdl_wait();                          // residual, output and state belong to the stream

    int tile_it = 0;
    bool stop = false;
    for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
      const TileCoord tc = tile_coord(p, pt);
      int my_px;
      if constexpr (SMALL) {
        // Column `lane` of this half: image n0 + 2*half + lane/16, row
        // (lane/4)%4, column lane%4 (4x4 images).
        const int n = tc.n0 + 2 * half + (lane >> 4);
        my_px = n < p.B ? (n * 4 + ((lane >> 2) & 3)) * 4 + (lane & 3) : -1;
      } else {
        const int col = half * 32 + lane;
        const int oh = tc.h0 + col / 8, ow = tc.w0 + (col & 7);
        my_px = (oh < p.OH && ow < p.OW) ? (tc.n0 * p.OH + oh) * p.OW + ow : -1;
      }
      int rows[4];
      store_rows(my_px, lane, rows);
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int px = __shfl_sync(0xffffffffu, my_px, i);
        v[i] = ((p.flags & kReadState) && cvalid && px >= 0)
                   ? p.state[static_cast<size_t>(px) * p.F + cout] : 0.f;
      }
      for (int t = 0; t < T; ++t) {
        const size_t tbase = static_cast<size_t>(t) * P;
        uint4 r4[4];
        if constexpr (RES) load_residual_rows(p.residual, tbase, rows, p.F, cbase, lane, chunk_ok, r4);
        bool fail = !mbar_wait_bounded(&acc_full[t], tile_it & 1, p.timeout_ns);
        fail = __any_sync(0xffffffffu, fail || *abort_flag);
        if (fail) { atomicOr(p.err, kErrTimeoutAcc); stop = true; break; }
        tc_fence_after();
        float acc[32];
        if (warp_live) {
          uint32_t r[32];
          if constexpr (SMALL) {
            // Image 2*half + j/4, row j%4 at timestep t: 4 columns each.
#pragma unroll
            for (int j = 0; j < 8; ++j)
              tmem_ld4_nowait(lane_base + 4 * (((j & 3) * 4 + 2 * half + (j >> 2)) * T + t), r + 4 * j);
          } else {
            // Output rows 4*half + j at timestep t: 8 columns each.
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tmem_ld8_nowait(lane_base + 8 * (T * (4 * half + j) + t), r + 8 * j);
          }
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[t]);              // the next tile's MMAs may reuse it
        if (!warp_live) continue;
        if constexpr (MODE == kModeNone) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int px = __shfl_sync(0xffffffffu, my_px, i);
            if (cvalid && px >= 0) p.out_f32[(tbase + px) * p.F + cout] = fmaf(acc[i], sc, bi);
          }
        } else {
          if (tma_out && n_st > 0) {
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
          }
#pragma unroll
          for (int i = 0; i < 32; ++i)
            xpose_put(xb, i, lane, neuron_step<MODE>(v[i], fmaf(acc[i], sx, bx), p.decay, p.tau,
                                                     p.v_th, p.v_reset));
          __syncwarp();
          if (tma_out) {
            if constexpr (RES) add_rows_into_xpose(xb, lane, r4);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if constexpr (SMALL) tma_store_5d(&p.tmap_out, xb, cbase, 0, 0, tc.n0 + 2 * half, t);
              else tma_store_5d(&p.tmap_out, xb, cbase, tc.w0, tc.h0 + 4 * half, tc.n0, t);
              bulk_commit_group();
            }
            ++n_st;
          } else {
            store_xpose_rows<RES>(p.out, xb, tbase, rows, p.F, cbase, lane, chunk_ok, r4);
            __syncwarp();
          }
        }
      }
      ++tile_it;
      if (!stop && (p.flags & kWriteState) && warp_live) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int px = __shfl_sync(0xffffffffu, my_px, i);
          if (cvalid && px >= 0) p.state[static_cast<size_t>(px) * p.F + cout] = v[i];
        }
      }
    }
    if (tma_out && lane == 0) bulk_wait_group<0>();   // stores complete before the CTA exits
    if (stop) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kHaloMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kHaloTmemCols);
  }
}

}  // namespace snn
