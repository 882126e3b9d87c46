/*
 * snn_b200.h -- C ABI of libsnnb200.so, the B200 (sm_100a) backend for the
 * fused 2:4-sparse Conv/Linear + BatchNorm + LIF/IF (+SEW residual add)
 * layer of SparseSNN's sengine.
 *
 * Plain pointers and sizes only.  Device pointers are CUDA global-memory
 * pointers; `stream` is a cudaStream_t passed as void*.  Every entry point
 * returns 0 on success and a negative SNN_E* code on failure; the message of
 * the last failure on the calling thread is available from
 * snn_last_error_message().  Kernel launches never allocate, synchronise or
 * change host state, so they may be captured into a CUDA graph.
 *
 * Tensor layouts (the reference's, sengine/kernels/interleaved_templates.py:95-154):
 *   data      [T*B][H][W][Cin]  fp16, NHWC, timestep-major
 *   out       [T*B][OH][OW][Cout] fp16 spikes (or spikes + residual),
 *             or fp32 BatchNorm output when neuron == SNN_NEURON_NONE
 *   state     [B*OH*OW][Cout]   fp32 membrane (read at start when
 *             SNN_FLAG_READ_STATE, final v written when SNN_FLAG_WRITE_STATE)
 *   bn_scale, bn_bias [Cout]    fp32, epilogue computes acc*scale + bias
 *             (the reference keeps BN out of the weights,
 *             sengine/optimizer.py:160-183)
 *   residual  [T*B][OH][OW][Cout] fp16 (SEW ADD identity, or the
 *             real-valued skip input of an Add that precedes the neuron)
 *   weight    packed 2:4 blob produced by snn_pack_weight_24
 */
#ifndef SNN_B200_H
#define SNN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SNN_ABI_VERSION 3

enum {
  SNN_OK = 0,
  SNN_E_INVALID = -1,      /* bad argument or unsupported geometry */
  SNN_E_NOT_24 = -2,       /* weight has a group of 4 with more than 2 non-zeros */
  SNN_E_CUDA = -3,         /* CUDA runtime / driver call failed */
  SNN_E_NO_DEVICE = -4,    /* no sm_100 device */
  SNN_E_DEVICE = -5        /* kernel reported a bounded-wait timeout */
};

/* Neuron after BN.  SNN_NEURON_NONE: fp32 BN output.  SNN_NEURON_NONE_F16:
 * fp16 BN output, and with a residual (snn_conv_forward_res, ADD_AFTER)
 * out = bn + residual, rounded once: the real-valued membrane-shortcut sum of
 * MS-ResNet (models/msresnet.py:119-123). */
enum { SNN_NEURON_LIF = 0, SNN_NEURON_IF = 1, SNN_NEURON_NONE = 2, SNN_NEURON_NONE_F16 = 3 };
enum { SNN_FLAG_READ_STATE = 1, SNN_FLAG_WRITE_STATE = 2,
       /* Always use the general kernel (streamed weights, per-tap activation
        * tiles) even where the halo kernel applies; for testing. */
       SNN_FLAG_FORCE_GENERIC = 4,
       /* Run eligible general-kernel layers (3x3, four-timestep 64-pixel
        * tiles, an even number of 128-channel tiles) on CTA pairs: 2-CTA
        * clusters sharing one M = 256 MMA, each CTA loading half of the
        * activations.  Measured 2-4 us faster per SEW-ResNet-18 stage-3/4
        * layer in isolation but not faster inside the whole-forward CUDA
        * graph, so it is not the default. */
       SNN_FLAG_CTA_PAIR = 8,
       /* Dense (unpruned) weights: the layer runs as the sum of two 2:4
        * layers over the same activations (weight positions 0,1 and 2,3 of
        * every group of four input channels), which the packer splits; the
        * packed blob holds 2*K weight columns.  General kernel only, spiking
        * neurons with no residual or the SEW add.  For dense convs the
        * reference keeps unpruned (e.g. a Spikformer's patch-splitting
        * convs, models/spikformer.py:159-206). */
       SNN_FLAG_DENSE = 16,
       /* Attention only: q, k and v are the three channel blocks of one
        * [T*B][N][3*heads*head_dim] tensor (rows of 3*C elements, as one
        * fused q|k|v Linear writes them); pass q, k = q + C and v = q + 2C. */
       SNN_FLAG_QKV_PACKED = 32,
       /* Bit-packed spikes: a [T*B][H][W][C] spike tensor stored as
        * [T*B][H][W][C/8] bytes, channel c in bit c%8 of byte c/8 (C a
        * multiple of 16).  Written by snn_stem_forward (LIF or IF neuron,
        * general tensor-core stem geometries), read by
        * snn_maxpool_lif_forward with SNN_NEURON_NONE (the pool after a
        * neuron, whose fp16 output is then the pooled spikes): an eighth of
        * the fp16 bytes between the two. */
       SNN_FLAG_SPIKE_BITS = 64 };

/* Where the residual of a fused Add enters the epilogue (the reference's
 * pattern strings and templates, sengine/kernels/interleaved_templates.py:371-397):
 *   ADD_AFTER   "Conv2d+LIF+Add": out = spike + residual (SEW ADD,
 *               conv1x1_bn_if_add, :230-288);
 *   ADD_BEFORE  "Conv2d+Add+LIF": the neuron integrates bn + residual
 *               (conv1x1_bn_add_lif, :163-221);
 *   TWO_NEURON  "Conv2d+IF+Add+LIF": s1 = neuron(bn); out = neuron2(s1 +
 *               residual), two membranes (conv1x1_bn_if_add_lif, :297-364);
 *               only through snn_conv_forward_res2. */
enum { SNN_RES_ADD_AFTER = 0, SNN_RES_ADD_BEFORE = 1, SNN_RES_TWO_NEURON = 2 };

/* One fused layer.  Linear layers are 1x1 convs over H=1, W=rows, B=1.
 * The fields after v_reset only matter for the residual entry points; a
 * zero-initialised tail selects the SEW ADD. */
typedef struct snn_conv_desc {
  int32_t T, B, Cin, H, W;
  int32_t Cout, KH, KW, stride, pad;
  int32_t neuron;            /* SNN_NEURON_* (the first neuron) */
  int32_t flags;             /* SNN_FLAG_* */
  float tau, v_threshold, v_reset;
  int32_t res_mode;          /* SNN_RES_* */
  int32_t neuron2;           /* TWO_NEURON: SNN_NEURON_LIF or SNN_NEURON_IF */
  float tau2, v_threshold2, v_reset2;
} snn_conv_desc;

/* Library ABI version (SNN_ABI_VERSION). */
int snn_abi_version(void);

/* Checks for an sm_100 device and resolves the driver's tensor-map encoder.
 * Replaces the per-kernel `int init(void)` of the reference's exported
 * TileLang .so (sengine/build/export_standalone.py:1-8, called by
 * sengine/csrc/cpp_executor.cu:637-652). */
int snn_init(void);

/* Kernel variants behind snn_conv_forward (all fused and numerically
 * equivalent up to fp32 accumulation order):
 *   GENERIC        streamed weights, one activation tile per filter tap
 *                  (also every ADD_BEFORE / TWO_NEURON residual layer);
 *   HALO_RESIDENT  stride-1 3x3, weights resident in shared memory, one
 *                  input halo per (timestep, 64-channel slice) shared by all taps;
 *   HALO_STREAM    stride-1 3x3 on images >= 8x8, T <= 4, streamed weights
 *                  reused across all timesteps, halo-shared taps. */
enum { SNN_VARIANT_GENERIC = 0, SNN_VARIANT_HALO_RESIDENT = 1, SNN_VARIANT_HALO_STREAM = 2 };

/* Variant snn_conv_forward will use for a descriptor (>= 0), or an error. */
int snn_conv_variant(const snn_conv_desc* d);

/* Output spatial size for a descriptor. */
int snn_conv_out_shape(const snn_conv_desc* d, int32_t* OH, int32_t* OW);

/* Bytes of the packed weight blob: compressed fp16 values [Cout_pad][K/2]
 * followed (256-byte aligned) by metadata words [Cout_pad/128][K/32][128],
 * where K = KH*KW*Cin_pad (Cin rounded up to 64: a layer's last 64-channel
 * block reads zeros past Cin; Cin must be a multiple of 8), doubled for
 * SNN_FLAG_DENSE. */
int snn_conv_weight_bytes(const snn_conv_desc* d, size_t* bytes);

/* Host-side 2:4 packer.  `w` is the pruned weight in the reference's
 * PyTorch layout [Cout][Cin][KH][KW] fp32 (host memory); groups of 4 run
 * along Cin inside each (kh,kw) tap (sengine/optimizer.py:499-523 order).
 * Writes snn_conv_weight_bytes() bytes to `blob` (host memory).
 * Returns SNN_E_NOT_24 if a group has more than 2 non-zeros. */
int snn_pack_weight_24(const snn_conv_desc* d, const float* w, void* blob);

/* Fused sparse conv + BN + neuron over T.  The 6-pointer + stream shape of
 * the reference's TileLang `call(data, weight, state, bn_scale, bn_bias,
 * out, stream)` (typedef TLCallFn6, sengine/csrc/sengine_exec.cu:443; call
 * site sengine/csrc/cpp_executor.cu:909-913), with the layer geometry passed
 * as a descriptor because one library serves every shape. */
int snn_conv_forward(const snn_conv_desc* d, const void* data, const void* weight,
                     float* state, const float* bn_scale, const float* bn_bias,
                     void* out, void* stream);

/* Same with a residual: d->res_mode SNN_RES_ADD_AFTER gives the SEW
 * out = spike + residual (the "LIF then Add" epilogue of
 * sengine/kernels/interleaved_templates.py:230-288, with LIF decay);
 * SNN_RES_ADD_BEFORE feeds bn + residual to the neuron (:163-221, with LIF
 * decay where the neuron is a LIF).  The reference executor cannot dispatch
 * either: it passes at most 6 arguments, sengine/csrc/cpp_executor.cu:895-914. */
int snn_conv_forward_res(const snn_conv_desc* d, const void* data, const void* weight,
                         float* state, const float* bn_scale, const float* bn_bias,
                         const void* residual, void* out, void* stream);

/* Two neurons around the Add (d->res_mode == SNN_RES_TWO_NEURON): s1 =
 * neuron(bn) with membrane `state`, out = neuron2(s1 + residual) with
 * membrane `state2` (same flags), fp16 spikes.  Argument order of the
 * reference template conv1x1_bn_if_add_lif (data, weight, state1, state2,
 * bn_scale, bn_bias, residual, output; interleaved_templates.py:297-364). */
int snn_conv_forward_res2(const snn_conv_desc* d, const void* data, const void* weight,
                          float* state, float* state2, const float* bn_scale,
                          const float* bn_bias, const void* residual, void* out,
                          void* stream);

/* Timestep-split form of the fused layer, for long T on few images (the
 * DVS configuration: T = 16, 4 images per GPU), where the one-pass kernels
 * have few pixel tiles to spread over the SMs because each CTA walks the T
 * chunks of its tiles in order.  Phase 1 runs conv + BN for all T*B images at
 * once (no neuron) into `workspace` as fp32; phase 2 runs the neuron over T
 * from there (+ the residual: d->res_mode ADD_AFTER or ADD_BEFORE, or
 * residual null) and writes the spikes.  Same arguments and results as
 * snn_conv_forward / snn_conv_forward_res (LIF or IF neuron, no dense weights)
 * plus a device workspace of at least snn_conv_tsplit_workspace_bytes()
 * bytes, 16-byte aligned, owned by the caller, reused across calls (out and
 * residual 16-byte aligned).  No
 * counterpart in the reference: its fused kernels keep the T loop inside one
 * CTA (sengine/kernels/conv2d_bn_if_t4.py:952-1020). */
int snn_conv_tsplit_workspace_bytes(const snn_conv_desc* d, size_t* bytes);
int snn_conv_forward_tsplit(const snn_conv_desc* d, const void* data, const void* weight,
                            float* state, const float* bn_scale, const float* bn_bias,
                            const void* residual, void* out, void* workspace,
                            size_t workspace_bytes, void* stream);

/* The timestep-split layer for callers that cannot allocate device memory
 * (a runtime that hands out every allocation from its own pool, or a process
 * where allocating is off limits once it serves): the fp32 intermediate lives
 * in a fixed array inside the library, SNN_TSPLIT_STATIC_MAX_BYTES per GPU,
 * held by every GPU that loads the library until the process exits.  Same
 * arguments and results as snn_conv_forward_tsplit without the workspace;
 * layers whose intermediate (snn_conv_tsplit_workspace_bytes) exceeds the
 * array are rejected with SNN_E_INVALID.  Allocates nothing.  The first call
 * on each device looks up the array's device address (with that device
 * current), so make that first call before any stream capture.  Calls share
 * the one array: two calls that overlap on the GPU (other streams, other
 * threads) race.  No counterpart in the reference. */
#define SNN_TSPLIT_STATIC_MAX_BYTES (8u << 20)
int snn_conv_forward_tsplit_static(const snn_conv_desc* d, const void* data, const void* weight,
                                   float* state, const float* bn_scale, const float* bn_bias,
                                   const void* residual, void* out, void* stream);

/* Dense direct-conv stem + BN + neuron (the Cin=3 first layer, which the
 * reference keeps dense: sengine/graph_slicer.py:106 skips Cin<4 and the
 * executor runs naive_conv2d_bn_nhwc_kernel, sengine/csrc/cpp_executor.cu:306-347).
 * x: [Tin][B][Cin][H][W] fp32 NCHW with Tin = 1 (input repeated over T,
 * models/sewresnet.py:199-201) or Tin = T.  w: [Cout][Cin][KH][KW] fp32.
 * out: [T][B][OH][OW][Cout] fp16 spikes, or with d->neuron ==
 * SNN_NEURON_NONE the fp16 BN output (MS-ResNet's stem feeds the real-valued
 * residual stream, models/msresnet.py:135-138,161).  With SNN_FLAG_SPIKE_BITS
 * in d->flags the spikes leave bit-packed, [T][B][OH][OW][Cout/8] bytes
 * (general tensor-core stem geometries only, as for snn_stem_forward_dual). */
int snn_stem_forward(const snn_conv_desc* d, int32_t Tin, const float* x, const float* w,
                     const float* bn_scale, const float* bn_bias, void* out, void* stream);

/* The stem without neuron followed by a standalone neuron node, in one pass:
 * out_bn gets the fp16 BN output (as snn_stem_forward with SNN_NEURON_NONE)
 * and out_spikes the spikes of d->neuron (LIF or IF, tau, v_threshold,
 * v_reset) run over T on that fp16 output, exactly as snn_lif_forward would
 * compute them from out_bn.  MS-ResNet's stem and the LIF in front of its
 * first block's conv (models/msresnet.py:119-121,135-138), which the
 * reference runs as the stem node plus lif_neuron_kernel
 * (sengine/csrc/cpp_executor.cu:46-64).  Both outputs [T][B][OH][OW][Cout]
 * fp16, 16-byte aligned; general tensor-core stem geometries only (Cout <=
 * 64, Cin*KH*KW <= 192), else SNN_E_INVALID. */
int snn_stem_forward_dual(const snn_conv_desc* d, int32_t Tin, const float* x, const float* w,
                          const float* bn_scale, const float* bn_bias, void* out_bn,
                          void* out_spikes, void* stream);

/* Classifier tail: global average pool over HW, mean over T, then
 * logits = feat @ fc_w^T + fc_b (models/sewresnet.py:207-210; the reference
 * executor runs global_avgpool, temporal_mean and a cuBLAS GEMM,
 * sengine/csrc/cpp_executor.cu:108-139,991-1016).
 * x: [T][B][HW][C] fp16; fc_w: [NC][C] fp32; fc_b: [NC] fp32; logits: [B][NC] fp32. */
int snn_head_forward(int32_t T, int32_t B, int32_t HW, int32_t C, int32_t NC,
                     const void* x, const float* fc_w, const float* fc_b, float* logits,
                     void* stream);

/* Fused Add + neuron over T: out = spikes of neuron(a + b) (the reference's
 * add_lif_fused_kernel, sengine/kernels/add_lif_fused.py:19-75, pattern
 * Add -> LIF, with the model's LIF/IF, models/neurons.py:121-146).
 * Shape from d: T, B, H, W and d->Cout channels (multiple of 8); neuron,
 * tau, v_threshold, v_reset and the state flags as for the conv.
 *   a, b   [T*B][H][W][C] fp16;   out [T*B][H][W][C] fp16 spikes
 *   state  [B*H*W][C] fp32 membrane */
int snn_add_lif_forward(const snn_conv_desc* d, const void* a, const void* b, float* state,
                        void* out, void* stream);

/* Fused MaxPool2d + neuron over T: out = spikes of neuron(maxpool(x)) (the
 * reference's maxpool_lif_fused_kernel, sengine/kernels/pool_lif_fused.py:
 * 15-79).  Window d->KH x d->KW, d->stride, d->pad (padding never wins the
 * max, as in torch MaxPool2d); channels d->Cin == d->Cout (multiple of 8).
 * d->neuron == SNN_NEURON_NONE gives the plain max pool (state unused): the
 * pool that follows a neuron, e.g. SEW-ResNet's stem maxpool
 * (models/sewresnet.py:202-203) or a Spikformer SPS pool
 * (models/spikformer.py:192-197).  That plain pool also reads bit-packed
 * spikes (SNN_FLAG_SPIKE_BITS in d->flags, C a multiple of 16, no state
 * flags): x is then [T*B][H][W][C/8] bytes and out the pooled fp16 spikes.
 *   x      [T*B][H][W][C] fp16;   out [T*B][OH][OW][C] fp16 spikes (or maxima)
 *   state  [B*OH*OW][C] fp32 membrane */
int snn_maxpool_lif_forward(const snn_conv_desc* d, const void* x, float* state, void* out,
                            void* stream);

/* Neuron over T of one input: out = spikes of neuron(x) (the reference
 * executor's standalone LIF node, lif_neuron_kernel,
 * sengine/csrc/cpp_executor.cu:46-64; in MS-ResNet the neuron in front of
 * every conv, models/msresnet.py:119-121).  Shape, neuron and state flags as
 * for snn_add_lif_forward.
 *   x      [T*B][H][W][C] fp16 (real-valued);   out same shape, fp16 spikes */
int snn_lif_forward(const snn_conv_desc* d, const void* x, float* state, void* out,
                    void* stream);

/* Spikformer attention core + attention LIF (the FusedSpikformerAttention op,
 * sengine/tdl/attention_ops.py:50-82 and :85-105; model semantics
 * models/spikformer.py:122-127 with attn_lif = MultiStepLIFNeuron(tau,
 * v_threshold), :97).  Per timestep and head: x = (q k^T * scale) v, then the
 * LIF over T with hard reset to v_reset.
 *   q, k, v  [T*B][N][heads*head_dim] fp16 spikes (0/1: the kernel forms
 *            q (k^T v) with k^T v rounded to fp16, exact for spikes), or with
 *            SNN_FLAG_QKV_PACKED the blocks of one [T*B][N][3*C] tensor
 *   out      [T*B][N][heads*head_dim] fp16 spikes
 *   state    [B][N][heads*head_dim] fp32 membrane, per SNN_FLAG_*_STATE
 * 1 <= N <= 256, head_dim 32 or 64.  x is exact (integer counts times scale)
 * for power-of-two scales such as the reference's 0.125. */
int snn_spikformer_attn_forward(int32_t T, int32_t B, int32_t N, int32_t heads,
                                int32_t head_dim, float scale, float tau, float v_threshold,
                                float v_reset, int32_t flags, const void* q, const void* k,
                                const void* v, float* state, void* out, void* stream);

/* Reads (and with reset != 0 clears) the device error word that kernels set
 * when a bounded wait times out.  Synchronises the device. */
int snn_get_device_error(uint32_t* code, int reset);

/* Message of the last failure on this thread ("" if none). */
const char* snn_last_error_message(void);

/* ------------------------------------------------------------------ engine
 * Whole-model executor over an engine file: a plan of fused nodes (stem,
 * sparse conv with optional residual, Add+LIF, MaxPool+LIF, head) in
 * execution order plus a packed parameter blob, as written by
 * sparsesnn_b200.engine_file.save_engine.  The loader validates the file,
 * allocates one device arena for every activation and uploads the
 * parameters; a forward is the node loop over the entry points above,
 * launched eagerly or replayed from a CUDA graph.  Membranes start at zero
 * every forward (single-call inference, as the reference executor after
 * sengine_reset_membranes, sengine/csrc/cpp_executor.cu:1196-1203). */
typedef struct snn_engine snn_engine;

/* Validates an engine file on the host (no device use) and reports its node
 * and tensor counts.  Replaces the parsing half of load_plan
 * (sengine/csrc/sengine_exec.cu:516) for this library's file layout. */
int snn_engine_check_file(const char* path, int32_t* n_nodes, int32_t* n_tensors);

/* Loads an engine file onto the current device (cudaMalloc of the activation
 * arena and the parameter blob).  Replaces load_plan
 * (sengine/csrc/sengine_exec.cu:516) and the per-node set-up calls of the
 * reference executor (sengine_create / sengine_set_*_node,
 * sengine/csrc/cpp_executor.cu:595-874). */
int snn_engine_load(const char* path, snn_engine** out);

/* Timesteps, batch, and byte sizes of the images ([B][C][H][W] fp32) and
 * logits ([B][classes] fp32) of a loaded engine. */
int snn_engine_io(const snn_engine* e, int32_t* T, int32_t* B, size_t* image_bytes,
                  size_t* logit_bytes);

/* Captures the node loop on `stream` (not the legacy default stream) into a
 * CUDA graph that later snn_engine_run calls replay
 * (sengine_capture_graph / sengine_replay, sengine/csrc/cpp_executor.cu:1270-1293). */
int snn_engine_capture(snn_engine* e, void* stream);

/* One forward on `stream` (sengine_execute, sengine/csrc/cpp_executor.cu:883-1194):
 * images (host or device, fp32) are copied into the engine's input buffer,
 * the nodes run (or the captured graph is replayed), and the logits are
 * copied to `logits` (host or device) -- all asynchronously on `stream`.
 * A host buffer must be pinned for the copies to overlap other work and
 * must stay valid until the stream reaches the copy.  images or logits may
 * be null to reuse / leave the engine's own buffers. */
int snn_engine_run(snn_engine* e, const float* images, float* logits, void* stream);

/* Frees the graph, the arena and the parameters (sengine_destroy,
 * sengine/csrc/cpp_executor.cu:609-629). */
void snn_engine_destroy(snn_engine* e);

#ifdef __cplusplus
}
#endif
#endif /* SNN_B200_H */
