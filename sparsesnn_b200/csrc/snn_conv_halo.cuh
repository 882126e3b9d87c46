// Halo variant of the fused 2:4-sparse conv for stride-1 KxK convolutions
// ("same" padding) whose per-tile weights fit in shared memory (e.g. 3x3
// with Cin <= 128).
//
// Differences from the generic kernel (snn_conv.cuh):
//  * the CTA's 128-channel weight slice (all k-blocks) is loaded ONCE into
//    shared memory and stays resident for the CTA's lifetime;
//  * a tile is 8 output columns x BN/8 output rows of one image; for each
//    (timestep, 64-channel slice) ONE TMA box loads the (8+K-1) x (BN/8+K-1)
//    input halo, and every filter tap reads it through a descriptor that
//    starts at row offset (kh*(8+K-1) + kw) with a group stride of one halo
//    row (the 128-byte swizzle is a function of the absolute shared-memory
//    address, so operands may start at any 128-byte row);
//  * timesteps are the outer loop; accumulators are double-buffered in
//    TMEM (2 x BN columns), and the epilogue copies a buffer to registers and
//    releases it before the neuron update.
//
// Warp roles (12 warps): 0..7 epilogue (TMEM lane quarter = warp % 4, pixel
// half = warp / 4); 8..11 load the metadata into TMEM (one warp per lane
// quarter), then warp 10 issues MMAs and owns TMEM and warp 11 drives TMA.
// Placing the MMA and TMA warps on sub-partitions 2 and 3 keeps them off the
// sub-partitions that do most of the epilogue work.
//
// M64 (layers with at most 64 output channels, BN = 128): the MMAs use M = 64,
// whose accumulator keeps 16 rows in each TMEM lane quarter (rows 16q..16q+15
// in lanes 32q..32q+15), so all eight epilogue warps hold real channels: warp
// (q, half) reads its 16 lanes x 64 columns with one 16x32bx2 load (thread t:
// channel 16q + t%16, 32 consecutive columns).  The 2:4 metadata of an M = 64
// MMA uses the same per-lane word format as M = 128, in lanes 32q..32q+15 for
// rows 16q..16q+15; the loader takes those words from M = 128 lanes 16q..16q+15
// of the packed blob.  Spikes go through a [64 px][64 ch] tile shared by the
// four warps of a half, so every warp store writes whole 128-byte pixel rows.
#pragma once
#include "snn_conv.cuh"

namespace snn {

constexpr int kHaloMaxStages = 8;
constexpr int kHaloThreads = 384;
constexpr int kHaloMmaWarp = 10;
constexpr int kHaloTmaWarp = 11;
constexpr int kHaloMetaCol = 256;        // accumulators: 2 x up to 128 columns
constexpr int kHaloTmemCols = 512;
constexpr int kHalo64TileBytes = 64 * 128;                 // [64 px][64 ch] fp16
constexpr int kHalo64XposeBytes = 4 * kHalo64TileBytes;    // 2 buffers x 2 halves
constexpr int kHaloXposeBytes = kEpiWarps * 2 * kXposeBytes;   // M = 128: 2 tiles per warp

struct HaloParams {
  ConvParams c;              // shared fields (tmap_a, tmap_b[0], meta, scale, ...)
  int KH;
  int halo_w;                // 8 + KW - 1 (pixels per halo row)
  int halo_bytes;            // bytes one halo box delivers
  int halo_stride;           // smem bytes per halo stage (1024-aligned)
  int halo_stages;
  int a_bytes;               // resident weight bytes (n_kb * kABytes)
};

// Byte offset of (pixel px, 16-byte channel chunk c16) in an M64 spike tile:
// 128-byte pixel rows, chunk index XOR-ed with 4 for pixels 32..63 so the two
// pixels one store instruction writes land in different banks.
__device__ __forceinline__ int tile64_off(int px, int c16) {
  return px * 128 + ((c16 ^ (((px >> 5) & 1) << 2)) << 4);
}

template <int MODE, bool RES, int BN, int KS, bool M64 = false>
__global__ void __launch_bounds__(kHaloThreads, 1)
fused_sparse_conv_halo_kernel(const __grid_constant__ HaloParams hp) {
  static_assert(!M64 || BN == 128, "the M = 64 path tiles 128 pixels");
  const ConvParams& p = hp.c;
  constexpr int G = BN / 64;                 // 32-column groups per epilogue warp
  constexpr int kAKb = (M64 ? 64 : kBM) * (kKB / 2) * 2;   // resident weight bytes per k-block
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                                              // resident weights
  uint8_t* sH = smem + hp.a_bytes;                                 // halo stages
  uint8_t* sX = sH + hp.halo_stages * hp.halo_stride;              // epilogue transposes
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + (M64 ? kHalo64XposeBytes : kHaloXposeBytes));
  uint64_t* empty = full + kHaloMaxStages;
  uint64_t* a_full = empty + kHaloMaxStages;
  uint64_t* acc_full = a_full + 1;          // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* meta_ready = acc_empty + 2;
  uint64_t* drain = meta_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int m_tile = blockIdx.x % p.n_m;
  const int first_pt = blockIdx.x / p.n_m;
  const int pt_step = gridDim.x / p.n_m;
  const int n_meta = 2 * p.n_kb;
  const int S = hp.halo_stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(a_full, 1);
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], kEpiThreads); }
    mbar_init(meta_ready, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kHaloTmaWarp && lane == 0) { prefetch_tmap(&p.tmap_a); prefetch_tmap(&p.tmap_b[0]); }
  if (warp == kHaloMmaWarp) { tmem_alloc(tmem_slot, kHaloTmemCols); tmem_relinquish(); }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kHaloTmaWarp && lane == 0) {
    // The whole resident weight slice is one 3-D box ([k-block][row][32
    // elements]), issued before anything else so that it lands while the
    // metadata loads below are in flight.
    mbar_arrive_expect_tx(a_full, hp.a_bytes);
    tma_load_3d(sA, &p.tmap_a, a_full, 0, m_tile * kBM, 0);
  }
  if (warp >= kEpiWarps) {
    // ------------------------------------------- metadata into TMEM (warps 8..11)
    const int q = warp & 3;
    // Blob lane whose words this TMEM lane takes (-1: unused by M = 64).
    const int row = M64 ? (lane < 16 ? q * 16 + lane : -1) : q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t* src = p.meta + (static_cast<size_t>(m_tile) * n_meta) * kBM + max(row, 0);
    // Up to 40 columns' loads in flight per lane (one round trip for every
    // resident-weight layer with at most 20 k-blocks).
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
          tmem_st8(lane_base + kHaloMetaCol + j + 8 * u, r8);
        }
      }
    }
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive(meta_ready);
  }

  if (warp == kHaloTmaWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      pdl_wait();                        // activations come from the previous kernel
      int stage = 0; uint32_t phase = 0;
      int issued = 0;
      bool stop = false;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        const TileCoord tc = tile_coord(p, pt);
        for (int t = 0; t < p.T && !stop; ++t) {
          for (int cb = 0; cb < p.cin_blocks; ++cb) {
            if (*abort_flag) { stop = true; break; }
            if (!mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutEmpty); *abort_flag = 1; stop = true; break;
            }
            mbar_arrive_expect_tx(&full[stage], hp.halo_bytes);
            tma_load_5d(sH + stage * hp.halo_stride, &p.tmap_b[0], &full[stage], cb * kKB,
                        tc.w0 - p.pad, tc.h0 - p.pad, tc.n0, t);
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
  } else if (warp == kHaloMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(M64 ? 64 : kBM, BN, true);
      bool ok = mbar_wait_bounded(meta_ready, 0, p.timeout_ns);
      ok = ok && mbar_wait_bounded(a_full, 0, p.timeout_ns);
      if (!ok) { atomicOr(p.err, kErrTimeoutMeta); *abort_flag = 1; }
      tc_fence_after();
      const uint32_t sbo = static_cast<uint32_t>(hp.halo_w) * 128;
      const uint64_t a_desc0 = smem_desc_kmajor(smem_u32(sA), 512, 4);
      const uint64_t h_desc0 = smem_desc_kmajor(smem_u32(sH), sbo, 2);
      const int halo_row16 = hp.halo_w * 8;            // one halo row of pixels, in 16-byte units
      int stage = 0; uint32_t phase = 0;
      int it = 0;
      bool stop = *abort_flag != 0;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        for (int t = 0; t < p.T && !stop; ++t) {
          const int buf = it & 1;
          if (!mbar_wait_bounded(&acc_empty[buf], ((it >> 1) & 1) ^ 1, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutAccEmpty); *abort_flag = 1; stop = true; break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + buf * BN;
          for (int cb = 0; cb < p.cin_blocks; ++cb) {
            if (!mbar_wait_bounded(&full[stage], phase, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutFull); *abort_flag = 1; stop = true; break;
            }
            tc_fence_after();
            // Descriptors advance by adding (byte offset >> 4) to the start
            // address field; the issue loop is the MMA thread's critical path.
            const uint64_t hd = h_desc0 + static_cast<uint32_t>(stage * hp.halo_stride >> 4);
#pragma unroll
            for (int kh = 0; kh < KS; ++kh) {
#pragma unroll
              for (int kw = 0; kw < KS; ++kw) {
                const int kb = (kh * KS + kw) * p.cin_blocks + cb;
                const uint64_t ad = a_desc0 + static_cast<uint32_t>(kb * (kAKb >> 4));
                const uint64_t bd = hd + static_cast<uint32_t>(kh * halo_row16 + kw * 8);
                const uint32_t e_addr = tmem + kHaloMetaCol + 2 * kb;
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                  const bool first = (cb == 0 && kh == 0 && kw == 0 && s == 0);
                  mma_sp_f16(d_tmem, ad + 2 * s, bd + 4 * s, e_addr, idesc | static_cast<uint32_t>(s),
                             first ? 0u : 1u);
                }
              }
            }
            mma_commit(&empty[stage]);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
          if (stop) break;
          mma_commit(&acc_full[buf]);
          ++it;
        }
      }
      mma_commit(drain);
      if (!mbar_wait_bounded(drain, 0, p.timeout_ns)) atomicOr(p.err, kErrTimeoutDrain);
    }
  } else if (M64 && warp < kEpiWarps) {
    // ------------------------------------------------------- epilogue, M = 64
    const int q = warp & 3;
    const int half = warp >> 2;
    const int ch = q * 16 + (lane & 15);         // this thread's output channel
    const bool cvalid = ch < p.F;
    const float sc = cvalid ? p.scale[ch] : 0.f;
    const float bi = cvalid ? p.bias[ch] : 0.f;
    const float sx = MODE == kModeLifHalf ? sc * 0.5f : sc;
    const float bx = MODE == kModeLifHalf ? bi * 0.5f : bi;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
    const int col0 = half * 64 + (lane >> 4) * 32;   // neuron phase: columns col0 + i
    const int tcol0 = (lane >> 4) * 32;              // ... as tile rows
    const int c16 = lane & 7;                        // row phase: 16-byte channel chunk
    const bool chunk_ok = c16 * 8 < p.F;
    const int bar_id = 1 + half;                     // named barrier of the half's 4 warps
    // Neuron phase: this thread writes tile rows tcol0 + i (i < 32), all with
    // bit 5 = lane/16, at byte (tcol0 + i)*128 + put_off.
    const int put_off = (((ch >> 3) ^ ((lane >> 4) << 2)) << 4) + (ch & 7) * 2;
    pdl_wait();                                      // residual, output and state

    int it = 0;
    bool stop = false;
    for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
      const TileCoord tc = tile_coord(p, pt);
      // Column j of the tile is pixel (h0 + j/8, w0 + j%8).
      auto px_of = [&](int col) -> int {
        const int oh = tc.h0 + col / 8, ow = tc.w0 + (col & 7);
        return (oh < p.OH && ow < p.OW) ? (tc.n0 * p.OH + oh) * p.OW + ow : -1;
      };
      // Row phase: this warp stores tile rows q*16 + 4j + lane/8 of its half.
      int rows[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) rows[j] = px_of(half * 64 + q * 16 + 4 * j + (lane >> 3));
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int px = px_of(col0 + i);
        v[i] = ((p.flags & kReadState) && cvalid && px >= 0)
                   ? p.state[static_cast<size_t>(px) * p.F + ch] : 0.f;
      }
      for (int t = 0; t < p.T; ++t) {
        const int buf = it & 1;
        const size_t tbase = static_cast<size_t>(t) * P;
        uint8_t* tile = sX + (buf * 2 + half) * kHalo64TileBytes;
        uint4 r4[4];
        if constexpr (RES) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            r4[j] = make_uint4(0, 0, 0, 0);
            if (chunk_ok && rows[j] >= 0)
              r4[j] = __ldg(reinterpret_cast<const uint4*>(p.residual + (tbase + rows[j]) * p.F) + c16);
          }
        }
        bool fail = !mbar_wait_bounded(&acc_full[buf], (it >> 1) & 1, p.timeout_ns);
        fail = __any_sync(0xffffffffu, fail || *abort_flag);
        if (!fail) {
          tc_fence_after();
          float acc[32];
          tmem_ld16x2_32(lane_base + buf * BN + half * 64, acc);
          tc_fence_before();
          mbar_arrive(&acc_empty[buf]);          // buffer drained: the next MMAs may start
          if constexpr (MODE == kModeNone) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int px = px_of(col0 + i);
              if (cvalid && px >= 0) p.out_f32[(tbase + px) * p.F + ch] = fmaf(acc[i], sc, bi);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const bool spike = neuron_step<MODE>(v[i], fmaf(acc[i], sx, bx), p.decay, p.tau,
                                                   p.v_th, p.v_reset);
              *reinterpret_cast<__half*>(tile + (tcol0 + i) * 128 + put_off) =
                  __ushort_as_half(spike ? 0x3C00 : 0);
            }
          }
        }
        ++it;
        // The four warps of this half agree on aborting and see each other's
        // tile rows; the next use of this tile buffer is two barriers away.
        if (named_barrier_or(bar_id, 128, fail)) { atomicOr(p.err, kErrTimeoutAcc); stop = true; break; }
        if constexpr (MODE != kModeNone) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 o = *reinterpret_cast<const uint4*>(tile + tile64_off(q * 16 + 4 * j + (lane >> 3), c16));
            if constexpr (RES) {
              __half2* a = reinterpret_cast<__half2*>(&o);
              const __half2* b = reinterpret_cast<const __half2*>(&r4[j]);
#pragma unroll
              for (int u = 0; u < 4; ++u) a[u] = __hadd2(a[u], b[u]);
            }
            if (chunk_ok && rows[j] >= 0)
              reinterpret_cast<uint4*>(p.out + (tbase + rows[j]) * p.F)[c16] = o;
          }
        }
      }
      if (!stop && (p.flags & kWriteState)) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int px = px_of(col0 + i);
          if (cvalid && px >= 0) p.state[static_cast<size_t>(px) * p.F + ch] = v[i];
        }
      }
    }
    if (stop) *abort_flag = 1;
  } else if (!M64 && warp < kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = warp >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int cout = m_tile * kBM + row;
    const bool cvalid = cout < p.F;
    const int cbase = m_tile * kBM + q * 32;
    const bool warp_live = cbase < p.F;          // warp-uniform: any channel to write?
    const float sc = cvalid ? p.scale[cout] : 0.f;
    const float bi = cvalid ? p.bias[cout] : 0.f;
    const float sx = MODE == kModeLifHalf ? sc * 0.5f : sc;
    const float bx = MODE == kModeLifHalf ? bi * 0.5f : bi;
    const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
    const int nchunk8 = max(0, min(4, (p.F - cbase) / 8));
    const bool chunk_ok = (lane & 3) < nchunk8;
    // Spikes leave through TMA stores of this warp's two transpose tiles
    // (alternating per 32-pixel group; the tile layout is the 64-byte TMA
    // swizzle of a {32 ch, 8 w, 4 h} box): global stores from the epilogue
    // warps would slow the MMAs' shared-memory operand reads.  Lane 0 issues
    // the stores and, before a tile is rewritten, waits until its previous
    // store has read it.
    uint8_t* xbuf = sX + warp * 2 * kXposeBytes;
    int n_groups = 0;
    pdl_wait();                          // residual, output and state belong to the stream

    int it = 0;
    bool stop = false;
    for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
      const TileCoord tc = tile_coord(p, pt);
      // Column j of the tile is pixel (h0 + j/8, w0 + j%8); this warp owns
      // columns [half*BN/2, half*BN/2 + BN/2) in G groups of 32; my_px[g] is
      // the pixel of the group's column `lane` (the store rows are derived
      // from it by shuffles where needed, to keep registers for the membrane).
      int my_px[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int col = half * (BN / 2) + g * 32 + lane;
        const int oh = tc.h0 + col / 8, ow = tc.w0 + (col & 7);
        my_px[g] = (oh < p.OH && ow < p.OW) ? (tc.n0 * p.OH + oh) * p.OW + ow : -1;
      }
      float v[G][32];
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int px = __shfl_sync(0xffffffffu, my_px[g], i);
          v[g][i] = ((p.flags & kReadState) && cvalid && px >= 0)
                        ? p.state[static_cast<size_t>(px) * p.F + cout] : 0.f;
        }
      }
      for (int t = 0; t < p.T; ++t) {
        const int buf = it & 1;
        const size_t tbase = static_cast<size_t>(t) * P;
        // Residual rows: group 0's are requested before the accumulator wait
        // (their latency hides behind the MMAs), group g+1's right after group
        // g's neuron update, when its accumulator registers are free.
        uint4 r4[G][4];
        if constexpr (RES) {
          int rows[4];
          store_rows(my_px[0], lane, rows);
          load_residual_rows(p.residual, tbase, rows, p.F, cbase, lane, chunk_ok, r4[0]);
        }
        bool fail = !mbar_wait_bounded(&acc_full[buf], (it >> 1) & 1, p.timeout_ns);
        fail = __any_sync(0xffffffffu, fail || *abort_flag);
        if (fail) { atomicOr(p.err, kErrTimeoutAcc); stop = true; break; }
        tc_fence_after();
        if (!warp_live) {                      // no channel of this warp is real
          tc_fence_before();
          mbar_arrive(&acc_empty[buf]);
          ++it;
          continue;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float acc[32];
          tmem_ld32(lane_base + buf * BN + half * (BN / 2) + g * 32, acc);
          if (g == G - 1) {                    // buffer drained: the MMAs it holds back may start
            tc_fence_before();
            mbar_arrive(&acc_empty[buf]);
            ++it;
          }
          if constexpr (MODE == kModeNone) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int px = __shfl_sync(0xffffffffu, my_px[g], i);
              if (cvalid && px >= 0) p.out_f32[(tbase + px) * p.F + cout] = fmaf(acc[i], sc, bi);
            }
          } else {
            uint8_t* xb = xbuf + (n_groups & 1) * kXposeBytes;
            if (n_groups >= 2) {                 // this tile's previous store has read it
              if (lane == 0) bulk_wait_group_read<1>();
              __syncwarp();
            }
#pragma unroll
            for (int i = 0; i < 32; ++i)
              xpose_put(xb, i, lane, neuron_step<MODE>(v[g][i], fmaf(acc[i], sx, bx), p.decay,
                                                       p.tau, p.v_th, p.v_reset));
            __syncwarp();
            if constexpr (RES) {
              add_rows_into_xpose(xb, lane, r4[g]);
              if (g + 1 < G) {
                int rows[4];
                store_rows(my_px[g + 1], lane, rows);
                load_residual_rows(p.residual, tbase, rows, p.F, cbase, lane, chunk_ok, r4[g + 1]);
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              // Columns half*BN/2 + 32g .. +31 of the tile: 4 rows x 8 columns.
              const int col = half * (BN / 2) + g * 32;
              tma_store_5d(&p.tmap_b[1], xb, cbase, tc.w0, tc.h0 + col / 8, tc.n0, t);
              bulk_commit_group();
            }
            ++n_groups;
          }
        }
      }
      if (!stop && (p.flags & kWriteState) && warp_live) {  // (membranes after the last timestep)
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int px = __shfl_sync(0xffffffffu, my_px[g], i);
            if (cvalid && px >= 0) p.state[static_cast<size_t>(px) * p.F + cout] = v[g][i];
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();        // stores complete before the CTA exits
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
