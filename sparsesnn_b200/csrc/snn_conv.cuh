// Fused 2:4-sparse implicit-GEMM Conv/Linear + BN + LIF/IF (+SEW add) over T
// timesteps for sm_100a.
//
// GEMM view (per tile):  D[cout, pixel] = W_sp[cout, k] * X[k, pixel]
//   A = compressed 2:4 weights (M = 128 output channels), K-major, 64B swizzle
//   B = activations (N = 64 output pixels per timestep), K-major, 128B swizzle;
//       one 64-channel slice of one filter tap per k-block, fetched by TMA from
//       the NHWC input; out-of-bounds zero fill provides the conv padding
//   D = FP32 accumulators in tensor memory (TMEM): TC timesteps x 64 columns
//       per buffer (see GenCfg)
//   E = 2:4 metadata, resident in TMEM for the CTA's whole K range
//
// Persistent CTAs: each CTA owns one 128-channel slice (so its metadata is
// loaded once) and walks a strided list of pixel tiles.
//
// Warp roles (12 warps): 0, 10 and 11 = TMA producers (pipeline fill i is issued
// by producer i % 3), 1 = TMEM owner + MMA issuer, 2..9 = epilogue: two warps
// per TMEM lane quarter, each owning 32 of the 64 pixel columns.  The epilogue applies BN, runs the LIF/IF recurrence over T
// with the membrane in registers, stages fp16 spikes in a per-warp transpose
// tile, adds the SEW residual and writes 16-byte vectors (see the store stage
// below).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include "snn_ptx.cuh"

namespace snn {

constexpr int kBM = 128;             // output channels per tile (UMMA M)
constexpr int kBN = 64;              // output pixels per timestep per tile (UMMA N)
constexpr int kKB = 64;              // logical K per k-block (one 128B activation row)
constexpr int kABytes = kBM * (kKB / 2) * 2;     // 8 KB compressed weights
constexpr int kBBytes = kBN * kKB * 2;           // 8 KB activations per timestep
constexpr int kMetaCol = 256;                    // metadata columns start here
constexpr int kTmemCols = 512;
constexpr int kMaxMetaCols = kTmemCols - kMetaCol;  // => K <= 8192
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = kEpiWarps * 32;
// TMA producers: warps 0, 10 and 11.  One thread issues tensor copies one
// after another (a few hundred cycles each, whatever the box size), so
// several producer warps, producer i filling pipeline stages i, i+3, ...,
// keep the boxes coming; twelve warps (three per SM sub-partition) keep the
// epilogue's register budget at 168.
constexpr int kProducers = 3;
constexpr int kThreads = (2 + kEpiWarps + kProducers - 1) * 32;
constexpr int kXposeBytes = 32 * 32 * 2;         // per-warp [32 px][32 cout] fp16 transpose
constexpr int kBarBytes = 512;

// Pipeline shapes of the general kernel, by timesteps per accumulator (TC):
//  * TC = 2: two TMEM accumulators of 2 x 64 columns (the epilogue of one
//    chunk of timesteps overlaps the next chunk's MMAs); stages of two
//    k-blocks, so each wait/commit pair of the MMA thread covers four MMAs;
//  * TC = 4: one accumulator of 4 x 64 columns and N = 256 MMAs (one per
//    k-block half for all four timesteps).  A sparse MMA whose A, B and
//    metadata all change costs about 120 cycles up to N = 128 but runs at
//    its operand rate (160 cycles) at N = 256, so this wins even though the
//    next tile's MMAs wait for the epilogue to drain the single accumulator.
//  * CG2 (TC = 4 only, on request): a CTA pair (2-CTA cluster) computes two
//    adjacent 128-channel tiles of the same pixels with one M = 256 MMA
//    issued by the leader; each CTA loads its own weights and HALF of the
//    activation box (two of the four timesteps), so a CTA moves 24 KB per
//    k-block instead of 40 KB (the one-CTA version's k-blocks are paced by
//    that L2-to-SM feed, ~550 cycles against 320 of MMA).  Measured: the
//    pair's k-blocks come every ~510 cycles (the MMA then reads the peer's
//    half of B across the pair), layers 2-4 us faster in isolation, no
//    faster inside the whole-forward graph.
//  * AD = 2 (dense weights): a dense layer runs as the sum of two 2:4 layers
//    over the same activations -- weight half 0 keeps positions 0,1 of every
//    group of four input channels, half 1 keeps positions 2,3 -- so each
//    activation k-block meets two compressed weight tiles (two MMAs with
//    their own metadata columns, one B operand).  The stage holds both
//    weight tiles; the activation bytes per MMA halve.
template <int TC, bool CG2 = false, int AD = 1>
struct GenCfg {
  static_assert(!CG2 || TC == 4, "CTA pairs use the four-timestep tiles");
  static_assert(AD == 1 || (AD == 2 && !CG2), "dense weights: one-CTA tiles");
  static constexpr int kTC = TC;
  static constexpr int kAD = AD;
  static constexpr int kNumAcc = TC == 4 ? 1 : 2;
  static constexpr int kStages = CG2 ? 8 : TC == 4 ? (AD == 2 ? 4 : 5) : (AD == 2 ? 3 : 4);
  static constexpr int kKbPerStage = TC == 4 ? 1 : 2;
  static constexpr int kBTs = CG2 ? TC / 2 : TC;     // timesteps of the box this CTA loads
  static constexpr int kStageBytes = kKbPerStage * (AD * kABytes + kBTs * kBBytes);
  static constexpr int kAccCols = kTC * kBN;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiWarps * kXposeBytes + kBarBytes + 1024;
  static_assert(kNumAcc * kAccCols <= kMetaCol, "accumulators overlap the metadata columns");
};

enum NeuronKind : int { kLIF = 0, kIF = 1, kNoNeuron = 2 };
// Epilogue variants (template parameter): LIF with tau == 2 (every scaling
// by 1/2 is exact, so the update folds into two FMAs with the reference's
// rounding), LIF with general tau (v*(1-1/tau) + x/tau, each op rounded),
// IF, BN output without neuron (fp32), and BN output without neuron in
// fp16 through the store tile (plus a real-valued residual when RM is
// kResAddAfter: out = bn + residual, rounded once).
enum EpiMode : int { kModeLifHalf = 0, kModeLifDiv = 1, kModeIf = 2, kModeNone = 3, kModeBnF16 = 4 };

// One neuron step.  x2 is the BN output pre-scaled for kModeLifHalf
// (acc*(scale/2) + bias/2 == (acc*scale + bias)/2 exactly) and the plain BN
// output otherwise.  Returns the spike; updates v (hard reset to v_reset).
template <int MODE>
__device__ __forceinline__ bool neuron_step(float& v, float x2, float decay, float tau,
                                            float v_th, float v_reset) {
  float h;
  if constexpr (MODE == kModeLifHalf) h = fmaf(v, 0.5f, x2);      // v*0.5 is exact
  else if constexpr (MODE == kModeLifDiv) h = __fadd_rn(__fmul_rn(v, decay), __fdiv_rn(x2, tau));
  else h = __fadd_rn(v, x2);
  // (h - v_th) >= 0 is the reference's test; without flush-to-zero it equals h >= v_th.
  const bool spike = h >= v_th;
  v = spike ? v_reset : h;
  return spike;
}
// Second neuron of the kResTwoNeuron epilogue (LIF with general tau, or IF;
// for tau = 2 the LIF form gives the same bits as the folded one).
__device__ __forceinline__ bool neuron2_step(float& v, float x, bool lif, float decay, float tau,
                                             float v_th, float v_reset) {
  const float h = lif ? __fadd_rn(__fmul_rn(v, decay), __fdiv_rn(x, tau)) : __fadd_rn(v, x);
  const bool spike = h >= v_th;
  v = spike ? v_reset : h;
  return spike;
}
// ------------------------------------------------------ epilogue store stage
// An epilogue warp owns 32 output channels (one per TMEM lane) x 32 pixel
// columns.  The neuron loop writes the warp's spikes column by column into a
// per-warp transpose tile ([32 px][32 ch] fp16 in 64-byte rows whose 16-byte
// chunks are XOR-ed with (px>>1)&3, so the column writes and the row reads
// are both conflict-free).  The tile leaves with four lanes per pixel: lane l
// stores 16-byte chunk l%4 of column 8j + l/4, so one warp store covers 8
// pixels x 64 contiguous bytes (8 cache lines instead of 32).  The SEW
// residual is read with the same lane mapping.
__device__ __forceinline__ int xpose_off(int px, int c8) {
  return px * 64 + ((c8 ^ ((px >> 1) & 3)) << 4);
}
// Spike of this lane's channel at column i.
__device__ __forceinline__ void xpose_put(uint8_t* xb, int i, int lane, bool spike) {
  *reinterpret_cast<__half*>(xb + xpose_off(i, lane >> 3) + (lane & 7) * 2) =
      __ushort_as_half(spike ? 0x3C00 : 0);
}
// A real value of this lane's channel at column i (rounded to fp16).
__device__ __forceinline__ void xpose_put_val(uint8_t* xb, int i, int lane, float x) {
  *reinterpret_cast<__half*>(xb + xpose_off(i, lane >> 3) + (lane & 7) * 2) = __float2half_rn(x);
}
// Residual of this lane's channel at column i, from a transpose tile that
// holds the residual rows in store layout (the same place xpose_put writes).
__device__ __forceinline__ float xpose_get(const uint8_t* xb, int i, int lane) {
  return __half2float(*reinterpret_cast<const __half*>(xb + xpose_off(i, lane >> 3) + (lane & 7) * 2));
}
// Residual rows (store layout, see load_residual_rows) into the tile.
__device__ __forceinline__ void xpose_put_rows(uint8_t* xb, int lane, const uint4 (&r4)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(xb + xpose_off(8 * j + (lane >> 2), lane & 3)) = r4[j];
}
// Adds the SEW residual rows (store layout, see load_residual_rows) into a
// transpose tile in place.
__device__ __forceinline__ void add_rows_into_xpose(uint8_t* xb, int lane, const uint4 (&r4)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4* d = reinterpret_cast<uint4*>(xb + xpose_off(8 * j + (lane >> 2), lane & 3));
    uint4 o = *d;
    __half2* a = reinterpret_cast<__half2*>(&o);
    const __half2* b = reinterpret_cast<const __half2*>(&r4[j]);
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = __hadd2(a[u], b[u]);
    *d = o;
  }
}
// Pixels this lane stores (columns 8j + lane/4), from each lane's pixel of
// column `lane` (-1 = outside the output).
__device__ __forceinline__ void store_rows(int my_px, int lane, int (&rows)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) rows[j] = __shfl_sync(0xffffffffu, my_px, 8 * j + (lane >> 2));
}
__device__ __forceinline__ void load_residual_rows(const __half* res, size_t tbase,
                                                   const int (&rows)[4], int F, int cbase,
                                                   int lane, bool chunk_ok, uint4 (&r4)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    r4[j] = make_uint4(0, 0, 0, 0);
    if (chunk_ok && rows[j] >= 0)
      r4[j] = __ldg(reinterpret_cast<const uint4*>(res + (tbase + rows[j]) * F + cbase) +
                    (lane & 3));
  }
}
template <bool RES>
__device__ __forceinline__ void store_xpose_rows(__half* out, const uint8_t* xb, size_t tbase,
                                                 const int (&rows)[4], int F, int cbase,
                                                 int lane, bool chunk_ok, const uint4 (&r4)[4]) {
  const int c8 = lane & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 o = *reinterpret_cast<const uint4*>(xb + xpose_off(8 * j + (lane >> 2), c8));
    if constexpr (RES) {
      __half2* a = reinterpret_cast<__half2*>(&o);
      const __half2* b = reinterpret_cast<const __half2*>(&r4[j]);
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = __hadd2(a[u], b[u]);
    }
    if (chunk_ok && rows[j] >= 0)
      reinterpret_cast<uint4*>(out + (tbase + rows[j]) * F + cbase)[c8] = o;
  }
}

enum ConvFlags : int { kReadState = 1, kWriteState = 2 };
// Residual epilogues of the general kernel (template parameter RM): none;
// out = spike + residual (SEW ADD); the neuron integrates bn + residual;
// two neurons, out = neuron2(neuron(bn) + residual).
enum ResMode : int { kResNone = 0, kResAddAfter = 1, kResAddBefore = 2, kResTwoNeuron = 3 };
enum ErrCode : unsigned { kErrTimeoutFull = 1u, kErrTimeoutEmpty = 2u, kErrTimeoutAcc = 4u,
                          kErrTimeoutMeta = 8u, kErrTimeoutAccEmpty = 16u, kErrTimeoutDrain = 32u,
                          kErrTimeoutRes = 64u };

struct ConvParams {
  CUtensorMap tmap_a;        // compressed weights [Fpad][K/2] fp16 (2D)
  CUtensorMap tmap_b[4];     // activations (C, W', H', B, T), one map per stride parity
  CUtensorMap tmap_out;      // spikes (F, OW, OH, B, T), box {32 ch, one half-tile of pixels, 1 t}
  const uint32_t* meta;      // [Fpad/128][K/32][128]
  const float* scale;        // [F]
  const float* bias;         // [F]
  float* state;              // [B*OH*OW][F] or null
  float* state2;             // second membrane (kResTwoNeuron), same layout
  __half* out;               // [T*B*OH*OW][F] fp16 spikes (+ residual)
  const __half* residual;    // [T*B*OH*OW][F] fp16 or null
  float* out_f32;            // [T*B*OH*OW][F] (neuron == kNoNeuron only)
  unsigned* err;             // device error word
  int F, KW, stride, pad;
  int n_kb, cin_blocks;      // k-blocks, 64-channel slices per tap
  int B, OH, OW, T;
  int tw, th, tn;            // tile extent (output coords) along w, h, image
  int tiles_w, tiles_h, n_px_tiles, n_m;
  int box_bytes;             // bytes of one activation TMA box (tw*th*tn*128)
  int flags;
  int tma_out;               // general kernel: spikes leave by TMA stores through tmap_out
  float decay, tau, inv_tau, v_th, v_reset;
  int n2_lif;                // kResTwoNeuron: second neuron is a LIF (else IF)
  float decay2, tau2, v_th2, v_reset2;
  unsigned long long timeout_ns;   // bounded-wait budget, in SM clock cycles
};

__device__ __forceinline__ int floordiv2(int d) { return (d - (d & 1)) / 2; }

struct TileCoord { int w0, h0, n0; };

__device__ __forceinline__ TileCoord tile_coord(const ConvParams& p, int pt) {
  TileCoord c;
  const int tw_i = pt % p.tiles_w;
  const int rest = pt / p.tiles_w;
  const int th_i = rest % p.tiles_h;
  const int tn_i = rest / p.tiles_h;
  c.w0 = tw_i * p.tw; c.h0 = th_i * p.th; c.n0 = tn_i * p.tn;
  return c;
}

template <int MODE, int RM, int TC, bool CG2 = false, int AD = 1>
__global__ void __launch_bounds__(kThreads, 1)
fused_sparse_conv_lif_kernel(const __grid_constant__ ConvParams p) {
  constexpr bool RES = RM != kResNone;
  constexpr bool SPIKING = MODE != kModeNone && MODE != kModeBnF16;
  static_assert(MODE != kModeNone || RM == kResNone, "a residual epilogue needs a neuron");
  static_assert(MODE != kModeBnF16 || RM == kResNone || RM == kResAddAfter,
                "fp16 BN output: plain or plus the residual");
  static_assert(!CG2 || (SPIKING && RM <= kResAddAfter), "CTA pairs: spiking, SEW or none");
  using Cfg = GenCfg<TC, CG2, AD>;
  constexpr int kBTs = Cfg::kBTs;
  constexpr int kTC = Cfg::kTC, kNumAcc = Cfg::kNumAcc, kStages = Cfg::kStages;
  constexpr int kKbPerStage = Cfg::kKbPerStage, kStageBytes = Cfg::kStageBytes;
  constexpr int kAccCols = Cfg::kAccCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // Stage s holds k-blocks (A: kKbPerStage x AD x kABytes; B: kKbPerStage x kTC x kBBytes).
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kKbPerStage * AD * kABytes;
  uint8_t* sX = smem + kStages * kStageBytes;                // kEpiWarps x kXposeBytes
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + kEpiWarps * kXposeBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;                      // [kNumAcc]
  uint64_t* acc_empty = acc_full + kNumAcc;                  // [kNumAcc]
  uint64_t* meta_ready = acc_empty + kNumAcc;
  uint64_t* drain = meta_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // CTA pairs: cluster c owns the 128-channel tiles 2*(c % pairs) + rank of
  // the pixel tiles c / pairs, c / pairs + clusters / pairs, ...
  uint32_t rank = 0;
  int m_tile, first_pt, pt_step;
  if constexpr (CG2) {
    rank = cluster_ctarank();
    const int n_pairs = p.n_m / 2, cl = blockIdx.x >> 1;
    m_tile = 2 * (cl % n_pairs) + static_cast<int>(rank);
    first_pt = cl / n_pairs;
    pt_step = (gridDim.x >> 1) / n_pairs;
  } else {
    m_tile = blockIdx.x % p.n_m;
    first_pt = blockIdx.x / p.n_m;
    pt_step = gridDim.x / p.n_m;
  }
  const int n_chunks = (p.T + kTC - 1) / kTC;
  const int n_meta = 2 * p.n_kb * AD;                          // sparse K steps (32 each)
  // Pair: one arrival per epilogue warp of both CTAs on the leader's barriers.
  constexpr int kEpiArrivals = CG2 ? 2 * kEpiWarps : kEpiThreads;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < kNumAcc; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], kEpiArrivals); }
    mbar_init(meta_ready, kEpiArrivals);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (CG2) cluster_sync();     // the peer's barriers exist before anything signals them
  // The leader's barriers in the cluster window (for the follower's signals).
  const uint32_t full_l = CG2 ? mapa_shared(smem_u32(full), 0) : 0u;
  const uint32_t acc_empty_l = CG2 ? mapa_shared(smem_u32(acc_empty), 0) : 0u;
  const uint32_t meta_ready_l = CG2 ? mapa_shared(smem_u32(meta_ready), 0) : 0u;
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmap_a);
    for (int i = 0; i < (p.stride == 2 ? 4 : 1); ++i) prefetch_tmap(&p.tmap_b[i]);
  }
  if (warp == 1) {
    if constexpr (CG2) { tmem_alloc_pair(tmem_slot, kTmemCols); tmem_relinquish_pair(); }
    else { tmem_alloc(tmem_slot, kTmemCols); tmem_relinquish(); }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || warp >= 2 + kEpiWarps) {
    // ----------------------------------------------------------- producers
    const int prod = warp == 0 ? 0 : warp - (1 + kEpiWarps);   // 0..kProducers-1
    if (lane == 0) {
      pdl_wait();                        // activations come from the previous kernel
      int stage = 0; uint32_t phase = 0;
      int seq = 0;                       // pipeline fill index (all producers)
      bool stop = false;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        const TileCoord tc = tile_coord(p, pt);
        for (int c = 0; c < n_chunks && !stop; ++c) {
          const int t0 = c * kTC;
          for (int kb0 = 0; kb0 < p.n_kb; kb0 += kKbPerStage, ++seq) {
            if (seq % kProducers != prod) {
              if (++stage == kStages) { stage = 0; phase ^= 1; }
              continue;
            }
            if (*abort_flag) { stop = true; break; }
            if (!mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutEmpty); *abort_flag = 1; stop = true; break;
            }
            // One activation box spans the chunk's kTC timesteps (a timestep
            // beyond T is outside the tensor: zero-filled, never read).
            const int nk = min(kKbPerStage, p.n_kb - kb0);
            if constexpr (CG2) {
              // The leader's barrier counts both CTAs' bytes.
              if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * nk * (kABytes + kBTs * p.box_bytes));
            } else {
              mbar_arrive_expect_tx(&full[stage], nk * (AD * kABytes + kTC * p.box_bytes));
            }
            for (int j = 0; j < nk; ++j) {
              const int kb = kb0 + j;
              if constexpr (CG2) {
                tma_load_2d_pair(sA + (stage * kKbPerStage + j) * kABytes, &p.tmap_a,
                                 full_l + stage * 8, kb * (kKB / 2), m_tile * kBM);
              } else {
#pragma unroll
                for (int h = 0; h < AD; ++h)   // weight k-block kb*AD + h meets activation k-block kb
                  tma_load_2d(sA + ((stage * kKbPerStage + j) * AD + h) * kABytes, &p.tmap_a,
                              &full[stage], (kb * AD + h) * (kKB / 2), m_tile * kBM);
              }
              const int tap = kb / p.cin_blocks;
              const int cb = kb - tap * p.cin_blocks;
              const int kh = tap / p.KW, kw = tap - kh * p.KW;
              int map = 0, hoff = kh - p.pad, woff = kw - p.pad;
              if (p.stride == 2) {
                map = (hoff & 1) * 2 + (woff & 1);
                hoff = floordiv2(hoff); woff = floordiv2(woff);
              }
              if constexpr (CG2)
                tma_load_5d_pair(sB + (stage * kKbPerStage + j) * kBTs * kBBytes, &p.tmap_b[map],
                                 full_l + stage * 8, cb * kKB, tc.w0 + woff, tc.h0 + hoff, tc.n0,
                                 t0 + kBTs * static_cast<int>(rank));
              else
                tma_load_5d(sB + (stage * kKbPerStage + j) * kTC * kBBytes, &p.tmap_b[map], &full[stage],
                            cb * kKB, tc.w0 + woff, tc.h0 + hoff, tc.n0, t0);
            }
            if (++stage == kStages) { stage = 0; phase ^= 1; }
          }
        }
      }
      // Let every load this producer issued land before the CTA can exit.
      // Only the last kStages fills can still be in flight, one per stage,
      // so waiting on their parity cannot alias an older phase.  (A pair's
      // follower signals the leader's barriers; the leader's drain covers
      // its loads, and the pair leaves together.)
      for (int back = max(0, seq - kStages); back < seq && (!CG2 || rank == 0); ++back) {
        if (back % kProducers != prod) continue;
        if (!mbar_wait_bounded(&full[back % kStages], (back / kStages) & 1, p.timeout_ns))
          atomicOr(p.err, kErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && (!CG2 || rank == 0)) {
      const uint32_t idesc = idesc_f16(kBM, kBN, true);
      const uint32_t idesc2 = idesc_f16(CG2 ? 2 * kBM : kBM, kTC * kBN, true);
      const bool merge_ts = p.box_bytes == kBBytes;   // tiles of exactly 64 pixels
      if constexpr (CG2) {
        // The pair's MMA needs 64-pixel tiles and whole four-timestep chunks
        // (the host launches it only then).
        if (!merge_ts || p.T % kTC) { atomicOr(p.err, kErrTimeoutMeta); *abort_flag = 1; }
      }
      const uint64_t a_desc0 = smem_desc_kmajor(smem_u32(sA), 512, 4);
      const uint64_t b_desc0 = smem_desc_kmajor(smem_u32(sB), 1024, 2);
      if (!mbar_wait_bounded(meta_ready, 0, p.timeout_ns)) {
        atomicOr(p.err, kErrTimeoutMeta); *abort_flag = 1;
      }
      tc_fence_after();
      int stage = 0; uint32_t phase = 0;
      int acc_iter = 0;
      bool stop = *abort_flag != 0;
      for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
        for (int c = 0; c < n_chunks && !stop; ++c) {
          const int tcn = min(kTC, p.T - c * kTC);
          const int buf = acc_iter % kNumAcc;
          const uint32_t use = static_cast<uint32_t>(acc_iter / kNumAcc);
          if (!mbar_wait_bounded(&acc_empty[buf], (use & 1) ^ 1, p.timeout_ns)) {
            atomicOr(p.err, kErrTimeoutAccEmpty); *abort_flag = 1; stop = true; break;
          }
          tc_fence_after();
          const uint32_t d_base = tmem + buf * kAccCols;
          for (int kb0 = 0; kb0 < p.n_kb; kb0 += kKbPerStage) {
            if (!mbar_wait_bounded(&full[stage], phase, p.timeout_ns)) {
              atomicOr(p.err, kErrTimeoutFull); *abort_flag = 1; stop = true; break;
            }
            tc_fence_after();
            const int nk = min(kKbPerStage, p.n_kb - kb0);
            for (int jh = 0; jh < nk * AD; ++jh) {
              const int j = jh / AD;
              const int kbw = (kb0 + j) * AD + (jh - j * AD);   // weight k-block
              // Descriptors advance by adding (byte offset >> 4) to the start
              // address field (shared-memory addresses stay below 2^18).
              const uint64_t ad = a_desc0 + (((stage * kKbPerStage * AD + jh) * kABytes) >> 4);
              const uint64_t bd = b_desc0 + (((stage * kKbPerStage + j) * kBTs * kBBytes) >> 4);
#pragma unroll
              for (int s = 0; s < 2; ++s) {
                const uint32_t ecol = kMetaCol + 2 * kbw + s;
                const uint32_t e_addr = tmem + (ecol & ~1u);
                const uint32_t acc = (kbw > 0 || s > 0) ? 1u : 0u;
                if constexpr (CG2) {
                  // Pair: M = 256 (this CTA's rows and the follower's), N = 256
                  // (this CTA's two timesteps, then the follower's two).
                  mma_sp_f16_pair(d_base, ad + 2 * s, bd + 4 * s, e_addr, idesc2 | (ecol & 1u), acc);
                } else if (merge_ts && tcn == kTC) {
                  // The chunk's timesteps' 64-pixel tiles are consecutive rows
                  // of the box: one N = kTC * 64 MMA covers them.
                  mma_sp_f16(d_base, ad + 2 * s, bd + 4 * s, e_addr, idesc2 | (ecol & 1u), acc);
                } else {
                  for (int tt = 0; tt < tcn; ++tt)
                    mma_sp_f16(d_base + tt * kBN, ad + 2 * s, bd + ((tt * p.box_bytes + 64 * s) >> 4),
                               e_addr, idesc | (ecol & 1u), acc);
                }
              }
            }
            if constexpr (CG2) mma_commit_pair(&empty[stage], 0x3);
            else mma_commit(&empty[stage]);
            if (++stage == kStages) { stage = 0; phase ^= 1; }
          }
          if (stop) break;
          if constexpr (CG2) mma_commit_pair(&acc_full[buf], 0x3);
          else mma_commit(&acc_full[buf]);
          ++acc_iter;
        }
      }
      // Drain: every MMA issued so far completes before TMEM is released.
      if constexpr (CG2) mma_commit_pair(drain, 0x1);
      else mma_commit(drain);
      if (!mbar_wait_bounded(drain, 0, p.timeout_ns)) atomicOr(p.err, kErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------- metadata + epilogue
    const int e = warp - 2;                      // 0..7
    const int q = warp & 3;                      // TMEM lane quarter of this warp
    const int half = e >> 2;                     // which 32 pixel columns
    const int row = q * 32 + lane;               // output channel within the tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    {
      // 2:4 metadata into TMEM before the first MMA: the two warps of a lane
      // quarter take half of the columns each, and a lane issues up to 40
      // loads before storing them, so the MMAs wait for a few global round
      // trips rather than one per 8 columns (a TMEM store orders the loads
      // after it).  Columns past n_meta get the all-zero pattern (0x4).
      constexpr int kChunk = 40;
      const uint32_t* src = p.meta + (static_cast<size_t>(m_tile) * n_meta) * kBM + row;
      const int hcols = (n_meta + 15) / 16 * 8;          // columns per warp, multiple of 8
      const int c_begin = half * hcols, c_end = c_begin + hcols;
      for (int j = c_begin; j < c_end; j += kChunk) {
        uint32_t r[kChunk];
#pragma unroll
        for (int i = 0; i < kChunk; ++i)
          r[i] = (j + i < n_meta && j + i < c_end) ? __ldg(src + static_cast<size_t>(j + i) * kBM)
                                                   : 0x44444444u;
#pragma unroll
        for (int u = 0; u < kChunk / 8; ++u) {
          if (j + 8 * u < c_end) {
            uint32_t r8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) r8[i] = r[8 * u + i];
            tmem_st8(lane_base + kMetaCol + j + 8 * u, r8);
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      if constexpr (CG2) {
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(meta_ready);
          else mbar_arrive_cluster(meta_ready_l);
        }
      } else {
        mbar_arrive(meta_ready);
      }
    }

    const int cout = m_tile * kBM + row;
    const bool cvalid = cout < p.F;
    const float sc = cvalid ? p.scale[cout] : 0.f;
    const float bi = cvalid ? p.bias[cout] : 0.f;
    const long long P = static_cast<long long>(p.B) * p.OH * p.OW;
    const int tile_px = p.tw * p.th;
    pdl_wait();                          // residual, output and state belong to the stream
    const int cbase = m_tile * kBM + q * 32;     // first output channel of this warp
    const int nchunk8 = max(0, min(4, (p.F - cbase) / 8));   // valid 8-channel chunks
    const bool chunk_ok = (lane & 3) < nchunk8;
    uint8_t* xb = sX + e * kXposeBytes;
    // With p.tma_out the transpose tile (the 64-byte TMA swizzle of a
    // {32 ch, 32 px} box) leaves through a TMA store issued by lane 0, which
    // waits for that store to read the tile before the tile is rewritten:
    // global stores from the epilogue warps would slow the MMAs' and TMA's
    // shared-memory traffic.
    const bool tma_out = p.tma_out != 0;
    int n_st = 0;

    auto pixel_of = [&](const TileCoord& tc, int col) -> int {
      const int dn = col / tile_px;
      const int rem = col - dn * tile_px;
      const int dh = rem / p.tw;
      const int dw = rem - dh * p.tw;
      const int n = tc.n0 + dn, oh = tc.h0 + dh, ow = tc.w0 + dw;
      if (dn >= p.tn || n >= p.B || oh >= p.OH || ow >= p.OW) return -1;
      return (n * p.OH + oh) * p.OW + ow;
    };

    int acc_iter = 0;
    bool stop = false;
    for (int pt = first_pt; pt < p.n_px_tiles && !stop; pt += pt_step) {
      const TileCoord tc = tile_coord(p, pt);
      // Lane l's pixel is column half*32 + l (neuron phase: lane = channel,
      // so the column's pixel comes by shuffle).
      const int my_px = pixel_of(tc, half * 32 + lane);
      // Origin of this half's 32 pixels as a TMA box (w, h, image).
      int bw0, bh0, bn0;
      {
        const int col = half * 32;
        const int dn = col / tile_px, rem = col - dn * tile_px;
        bn0 = tc.n0 + dn; bh0 = tc.h0 + rem / p.tw; bw0 = tc.w0 + rem % p.tw;
      }
      int rows[4];
      store_rows(my_px, lane, rows);
      float v[32];
      float v2[RM == kResTwoNeuron ? 32 : 1];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int px = __shfl_sync(0xffffffffu, my_px, i);
        const bool rd = (p.flags & kReadState) && cvalid && px >= 0;
        v[i] = rd ? p.state[static_cast<size_t>(px) * p.F + cout] : 0.f;
        if constexpr (RM == kResTwoNeuron)
          v2[i] = rd ? p.state2[static_cast<size_t>(px) * p.F + cout] : 0.f;
      }
      for (int c = 0; c < n_chunks && !stop; ++c) {
        const int t0 = c * kTC;
        const int tcn = min(kTC, p.T - t0);
        const int buf = acc_iter % kNumAcc;
        const uint32_t use = static_cast<uint32_t>(acc_iter / kNumAcc);
        // Residual rows of the first two timesteps, fetched before the wait so
        // their latency overlaps the MMAs.
        uint4 r4[2][4];
        if constexpr (RES) {
#pragma unroll
          for (int u = 0; u < 2; ++u)
            if (u < tcn)
              load_residual_rows(p.residual, static_cast<size_t>(t0 + u) * P, rows, p.F, cbase, lane,
                                 chunk_ok, r4[u]);
        }
        bool fail = !mbar_wait_bounded(&acc_full[buf], use & 1, p.timeout_ns);
        fail = __any_sync(0xffffffffu, fail || *abort_flag);
        if (fail) { atomicOr(p.err, kErrTimeoutAcc); stop = true; break; }
        tc_fence_after();
        // Timesteps in pairs: both accumulators of a pair come in one TMEM
        // round trip; the buffer is released once its last pair is loaded.
        for (int t2 = 0; t2 < tcn; t2 += 2) {
          const int np = min(2, tcn - t2);
          uint32_t accr[2][32];
          tmem_ld32_nowait(lane_base + buf * kAccCols + t2 * kBN + half * 32, accr[0]);
          if (np > 1) tmem_ld32_nowait(lane_base + buf * kAccCols + (t2 + 1) * kBN + half * 32, accr[1]);
          tmem_wait_ld();
          if (t2 + 2 >= tcn) {                 // buffer drained: the MMAs it holds back may start
            tc_fence_before();
            if constexpr (CG2) {
              __syncwarp();
              if (lane == 0) {
                if (rank == 0) mbar_arrive(&acc_empty[buf]);
                else mbar_arrive_cluster(acc_empty_l + buf * 8);
              }
            } else {
              mbar_arrive(&acc_empty[buf]);
            }
          }
          if constexpr (RES) {
            if (t2 > 0) {                      // later pairs: fetched now, used after the update
#pragma unroll
              for (int u = 0; u < 2; ++u)
                if (u < np)
                  load_residual_rows(p.residual, static_cast<size_t>(t0 + t2 + u) * P, rows, p.F,
                                     cbase, lane, chunk_ok, r4[u]);
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (u >= np) break;
            const size_t tbase = static_cast<size_t>(t0 + t2 + u) * P;
            if constexpr (MODE == kModeNone) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int px = __shfl_sync(0xffffffffu, my_px, i);
                if (cvalid && px >= 0)
                  p.out_f32[(tbase + px) * p.F + cout] = fmaf(__uint_as_float(accr[u][i]), sc, bi);
              }
            } else {
              // Neuron update, lane = output channel, i = pixel column.
              const float sx = MODE == kModeLifHalf ? sc * 0.5f : sc;
              const float bx = MODE == kModeLifHalf ? bi * 0.5f : bi;
              if (tma_out && n_st > 0) {       // the tile's previous store has read it
                if (lane == 0) bulk_wait_group_read<0>();
                __syncwarp();
              }
              if constexpr (RM == kResAddBefore || RM == kResTwoNeuron ||
                            (MODE == kModeBnF16 && RM == kResAddAfter)) {
                // The residual enters the neuron (or the real-valued sum):
                // its rows go through the transpose tile, each lane reads its
                // channel per column and the result overwrites that same half.
                xpose_put_rows(xb, lane, r4[u]);
                __syncwarp();
              }
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                float x = fmaf(__uint_as_float(accr[u][i]), sx, bx);
                if constexpr (MODE == kModeBnF16) {
                  // No neuron: bn (+ residual) in fp32, rounded to fp16 once.
                  if constexpr (RM == kResAddAfter) x = __fadd_rn(x, xpose_get(xb, i, lane));
                  xpose_put_val(xb, i, lane, x);
                  continue;
                }
                if constexpr (RM == kResAddBefore) {
                  // kModeLifHalf: x is bn/2, and bn/2 + r/2 rounds to exactly
                  // (bn + r)/2, the folded form of the neuron's input.
                  const float r = xpose_get(xb, i, lane);
                  x = __fadd_rn(x, MODE == kModeLifHalf ? r * 0.5f : r);
                }
                bool spike = neuron_step<MODE>(v[i], x, p.decay, p.tau, p.v_th, p.v_reset);
                if constexpr (RM == kResTwoNeuron) {
                  const float x2 = __fadd_rn(spike ? 1.f : 0.f, xpose_get(xb, i, lane));
                  spike = neuron2_step(v2[i], x2, p.n2_lif != 0, p.decay2, p.tau2, p.v_th2,
                                       p.v_reset2);
                }
                xpose_put(xb, i, lane, spike);
              }
              __syncwarp();
              if (tma_out) {
                if constexpr (RM == kResAddAfter && MODE != kModeBnF16) add_rows_into_xpose(xb, lane, r4[u]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  tma_store_5d(&p.tmap_out, xb, cbase, bw0, bh0, bn0, t0 + t2 + u);
                  bulk_commit_group();
                }
                ++n_st;
              } else {
                store_xpose_rows<RM == kResAddAfter && MODE != kModeBnF16>(p.out, xb, tbase, rows, p.F,
                                                                           cbase, lane, chunk_ok, r4[u]);
                __syncwarp();
              }
            }
          }
        }
        ++acc_iter;
      }
      if (!stop && (p.flags & kWriteState)) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int px = __shfl_sync(0xffffffffu, my_px, i);
          if (cvalid && px >= 0) {
            p.state[static_cast<size_t>(px) * p.F + cout] = v[i];
            if constexpr (RM == kResTwoNeuron) p.state2[static_cast<size_t>(px) * p.F + cout] = v2[i];
          }
        }
      }
    }
    if (tma_out && lane == 0) bulk_wait_group<0>();   // stores complete before the CTA exits
    if (stop) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (CG2) cluster_sync();     // the leader's MMAs no longer read the follower's tiles
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG2) tmem_dealloc_pair(tmem, kTmemCols);
    else tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace snn
