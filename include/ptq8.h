/*
 * ptq8.h - C ABI of the B200-native (sm_100a) W8A8 / W4A8 quantized-conv engine.
 *
 * Drop-in boundary for the reference's int8 engine (PaperTigerL/ptq-int8-lab,
 * 06-gpu-int8/cpp).  Each entry point names the reference interface it
 * replaces.  Conventions: plain pointers and sizes; no entry point exits the
 * process (the reference's CUDA_CHECK calls std::exit, int8_engine.cuh:109-117);
 * every failure returns a nonzero status and the message is available from
 * ptq8_engine_last_error() or the caller's err buffer.  The engine owns its
 * device memory; the caller owns input / logits buffers and may provide the
 * CUDA stream.  One engine per device per host thread.
 */
#ifndef PTQ8_H
#define PTQ8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PTQ8_ABI_VERSION 1

/* status codes */
#define PTQ8_OK 0
#define PTQ8_ERR_INVALID 1  /* bad argument / state / unsupported topology */
#define PTQ8_ERR_FORMAT 2   /* malformed PTQ2 / PTQW / PTQC file */
#define PTQ8_ERR_CUDA 3     /* CUDA runtime error */
#define PTQ8_ERR_TIMEOUT 4  /* a bounded device wait ran out; outputs invalid */

/* graph passes (ptq8_engine_build `passes` bit mask) */
#define PTQ8_PASS_CENTER_TAP 1 /* 07-tensorrt-deploy/scripts/push_optimize_onnx.py:36-93 */
#define PTQ8_PASS_DECOMPOSE 2  /* 07-tensorrt-deploy/scripts/push_decompose.py:99-202  */
/* generalised positional decomposition: per-position sub-convs of convs whose output
 * positions read different kernel slices (push_decompose.py:50-80 computes the slices; its
 * decompose() declines such geometries); taps that only read padding are skipped */
#define PTQ8_PASS_POSITIONAL 4

/* activation range modes (06-gpu-int8/cpp/ptq_quant.h:163) */
#define PTQ8_ACT_ABSMAX 0
#define PTQ8_ACT_MINMAX 1

typedef struct ptq8_model ptq8_model;
typedef struct ptq8_engine ptq8_engine;

int ptq8_abi_version(void);

/* ---- calibrated-model files ------------------------------------------------ */

/* Model::load(path, err) - 06-gpu-int8/cpp/ptq_model.h:72-91.
 * PTQW or PTQ2 by magic, strict EOF, topology validation (ptq_model.h:104-203);
 * also PTQ8, this engine's native package (weight codes, f32 scales and bits per conv,
 * W4 two codes per byte; layout in csrc/ptq8_model.hpp), which builds without
 * re-quantizing.  Returns NULL on failure with the reason in err. */
ptq8_model* ptq8_model_load(const char* path, char* err, size_t errlen);
void ptq8_model_free(ptq8_model* m);

/* Counters of Model (ptq_model.h:65-70,205-229): out[11] = {n_conv, n_block,
 * stem_pool, fc_in, fc_out, n_depthwise, n_grouped, n_relu6, n_residual2,
 * format (1 PTQW, 2 PTQ2, 3 PTQ8), convs per block}. */
int ptq8_model_info(const ptq8_model* m, int* out);
/* ConvSpec of conv i (ptq_model.h:46-55): {cout, cin, kh, kw, sh, sw, ph, pw, relu, groups}. */
int ptq8_model_conv(const ptq8_model* m, int i, int* meta10);
/* BlockSpec of block i (ptq_model.h:57-63). */
int ptq8_model_block(const ptq8_model* m, int i, int* convs, int cap, int* n_convs, int* ds, int* stride,
                     int* residual);
/* Borrowed pointers to conv i's fp32 weight/bias (i = -1: the FC).  A PTQ8 conv has no
 * fp32 weights (n_weight 0). */
int ptq8_model_weights(const ptq8_model* m, int i, const float** weight, size_t* n_weight, const float** bias);
/* Borrowed pointers to conv i's stored codes ([cout][cin*kh*kw], one per byte) and f32
 * per-channel scales, and its bits (8 / 4), from a PTQ8 package; bits 0 and NULL
 * pointers for a PTQ2 / PTQW conv.  No counterpart in the reference (its files hold fp32
 * weights that Int8Engine::build quantizes, int8_engine.cuh:208). */
int ptq8_model_codes(const ptq8_model* m, int i, const int8_t** codes, size_t* n_codes, const float** scales,
                     int* bits);

/* load_ptqc(path, n_expected, out, err) - 06-gpu-int8/cpp/ptq_model.h:425-503.
 * Writes n (lo, hi) pairs to lohi[2n] (cap = number of floats available). */
int ptq8_load_ptqc(const char* path, size_t n_expected, float* lohi, size_t cap, char* err, size_t errlen);

/* tensor_quant_from_range scale (ptq_quant.h:195-214), returned in float64 as the
 * reference oracle uses it (09-ptq-toolkit/ptq_toolkit/ref_int8.py:69-87). */
double ptq8_act_scale(float lo, float hi, int bits, int mode);
/* quantize_weight_per_channel_sym (ptq_quant.h:72-110): w[cout][k] -> codes, f32 scales. */
int ptq8_quantize_weight(const float* w, int cout, int k, int bits, int8_t* codes, float* scale32);

/* Activation codes computed on `device` by the engine's own device quantizer
 * (the epilogue path): codes[i] = clip(round_half_away(double(x[i]) / s), -128, 127)
 * with s = ptq8_act_scale(lo, hi, 8, mode) (ref_int8.py:89-91).  Test entry point.
 * The range is checked like load_ptqc checks PTQC entries (ptq_model.h:425-503):
 * non-finite lo/hi, lo > hi, or a mode other than PTQ8_ACT_ABSMAX / PTQ8_ACT_MINMAX
 * return PTQ8_ERR_INVALID before any device work. */
int ptq8_quantize_device(int device, const float* x_host, size_t n, float lo, float hi, int mode, int8_t* codes);

/* Same codes as ptq8_quantize_device, but the call allocates no device memory
 * (no cudaMalloc / cudaFree, no allocating library routine).  No counterpart in
 * the reference.  For callers that cannot allocate: a process whose free device
 * memory is held by another allocator (a framework's caching pool, a serving
 * process at its memory cap) where a cudaMalloc may fail, and code that cannot
 * take the device-wide synchronisation cudaFree implies while other streams run.
 *
 * The input and output stay the caller's host buffers.  The device staging for
 * them is a fixed array inside the library, one per device, holding at most
 * PTQ8_NOALLOC_MAX_VALUES values (4 MiB of floats + 1 MiB of codes); a larger n
 * is rejected with PTQ8_ERR_INVALID and a message in err, and so is a range or mode
 * that ptq8_quantize_device rejects.  Every call looks the array's device address up
 * (cudaGetSymbolAddress, with the device current), so the first call on a device
 * loads the module there: make it before any stream capture.  All calls on a device
 * share the array and leave their data in it, so calls that overlap in time (two host
 * threads on the same device) race and must be serialised by the caller.  Copies and
 * the kernel run on the legacy default stream; the call returns when the codes are on
 * the host.  err (may be NULL) receives "" on success. */
#define PTQ8_NOALLOC_MAX_VALUES (1u << 20)
int ptq8_quantize_device_noalloc(int device, const float* x_host, size_t n, float lo, float hi, int mode,
                                 int8_t* codes, char* err, size_t errlen);

/* ---- engine ---------------------------------------------------------------- */

/* Int8Engine construction on CUDA device `device` (int8_engine.cuh:130). */
ptq8_engine* ptq8_engine_create(int device);
void ptq8_engine_destroy(ptq8_engine* e);
const char* ptq8_engine_last_error(const ptq8_engine* e);

/* Int8Engine::build(model, w_bits, a_bits) - int8_engine.cuh:132-349.
 * layer_bits (nullable, n_layer_bits == n_conv): per-conv weight bits 8/4 from a
 * layer plan (09-ptq-toolkit/ptq_toolkit/quant/mixed.py:126-212).  `passes` is a
 * PTQ8_PASS_* mask applied to the quantized layers.  The model must outlive the
 * engine (the reference keeps a raw pointer, int8_engine.cuh:134). */
int ptq8_engine_build(ptq8_engine* e, const ptq8_model* m, int w_bits, int a_bits, const int* layer_bits,
                      int n_layer_bits, int passes);
/* Int8Engine::set_act_mode - int8_engine.cuh:353. */
int ptq8_engine_set_act_mode(ptq8_engine* e, int mode);
/* Int8Engine::set_calib(ranges) - int8_engine.cuh:362-406; lohi[2n]. */
int ptq8_engine_set_calib(ptq8_engine* e, const float* lohi, size_t n);
/* Network input geometry (default 3x32x32, ptq_model.h:104 validates with 32x32). */
int ptq8_engine_set_input_shape(ptq8_engine* e, int c, int h, int w);
/* Int8Engine::alloc_scratch(n) - int8_engine.cuh:807-833: plan the launches and
 * allocate every activation buffer for batches up to max_batch. */
int ptq8_engine_alloc_scratch(ptq8_engine* e, int max_batch);
/* Int8Engine::set_stream - int8_engine.cuh:771 (NULL: engine-owned stream). */
int ptq8_engine_set_stream(ptq8_engine* e, void* stream);
/* Cap the persistent grid of every tensor-core conv at max_ctas CTAs (0: one per SM,
 * the default) -- e.g. to leave SMs to other work.  No counterpart in the reference
 * (its kernels are launched per tile).  Drops captured graphs. */
int ptq8_engine_set_max_ctas(ptq8_engine* e, int max_ctas);
void* ptq8_engine_stream(ptq8_engine* e);

/* Int8Engine::forward(x_host, n, c, h, w, logits_host) - int8_engine.cuh:429-645.
 * Host buffers: H2D, the whole forward as one CUDA graph, D2H, synchronize. */
int ptq8_engine_forward(ptq8_engine* e, const float* x_host, int n, int c, int h, int w, float* logits_host);
/* Pipelined host-buffer forward (no counterpart in the reference, whose forward is
 * synchronous): enqueues the H2D copy of x_host into one of two engine input slots on
 * an engine-owned copy stream, the forward (CUDA graph) on the engine stream once that
 * copy has landed, and the D2H copy of the logits; returns without waiting.  The H2D of
 * call k+1 overlaps the forward of call k.  ptq8_engine_sync() waits for every enqueued
 * call.  x_host (pinned, for the copies to overlap) must stay unchanged and logits_host
 * unread until then.  Same logits as ptq8_engine_forward.  The engine's other calls
 * that take or run on an input (forward, forward_device, run, input_buffer, profile,
 * ptq8_forward / ptq8_forward_debug) first wait for pipelined copies still in flight. */
int ptq8_engine_forward_async(ptq8_engine* e, const float* x_host, int n, float* logits_host);
/* Device-pointer forward (fp32 NCHW input, fp32 [n][fc_out] logits); enqueued
 * on the engine stream, not synchronized. */
int ptq8_engine_forward_device(ptq8_engine* e, const float* x_dev, int n, float* logits_dev);
/* ---- 8-bit pixel input (CIFAR-10 records) ----------------------------------
 * The reference decodes CIFAR-10 records and normalises them on the host, then
 * uploads fp32 (ref_e2e.py:261-276; main.cpp:178-198,245-261).  These calls upload the
 * 8-bit pixels (1 byte per value instead of 4) and the stem kernel does the
 * normalisation and the exact quantization on the device: the same network input
 * codes, bit for bit, as the reference's fp32 path, given the same normalisation.
 * Pixels are [n][c][h][w] bytes per image; image i starts at x + i * record_bytes
 * (record_bytes 0: c*h*w, packed; a raw CIFAR-10 batch file is x = file + 1,
 * record_bytes = 3073, skipping each record's label byte).  At most 4 channels. */
#define PTQ8_NORM_DIV 0 /* x = (px - mean*255) / (std*255): ref_e2e.py:272-274 (the default) */
#define PTQ8_NORM_MUL 1 /* x = ((px/255)*255 - mean*255) * (1/(std*255)): main.cpp:245-261 */
/* Normalisation of 8-bit input (mode PTQ8_NORM_*; mean/std: float[c], or both NULL for the
 * CIFAR-10 constants of main.cpp:25-26).  Every operation in float32, rounded to nearest.
 * Drops captured 8-bit-input graphs. */
int ptq8_engine_set_input_norm(ptq8_engine* e, int mode, const float* mean, const float* std_);
/* Int8Engine::forward (int8_engine.cuh:429) from 8-bit host pixels: H2D of the pixels,
 * the forward as one CUDA graph, D2H of the logits, synchronize. */
int ptq8_engine_forward_u8(ptq8_engine* e, const uint8_t* x_host, int n, size_t record_bytes, float* logits_host);
/* Pipelined form of ptq8_engine_forward_u8, with the semantics of ptq8_engine_forward_async
 * (same two input slots and copy stream; wait with ptq8_engine_sync). */
int ptq8_engine_forward_u8_async(ptq8_engine* e, const uint8_t* x_host, int n, size_t record_bytes,
                                 float* logits_host);
/* Device-pointer form (8-bit pixels on the device, fp32 logits [n][fc_out]); enqueued on
 * the engine stream, not synchronized. */
int ptq8_engine_forward_device_u8(ptq8_engine* e, const uint8_t* x_dev, int n, size_t record_bytes,
                                  float* logits_dev);

/* Engine-resident buffers: callers may write inputs straight into the input
 * buffer and run ptq8_engine_run() with no copies. */
float* ptq8_engine_input_buffer(ptq8_engine* e);
float* ptq8_engine_logits_buffer(ptq8_engine* e);
int ptq8_engine_run(ptq8_engine* e, int n, int use_graph);
/* Async device-to-device copy of the last forward's logits ([n][fc_out]) on the engine stream. */
int ptq8_engine_copy_logits(ptq8_engine* e, int n, float* dst_dev);
int ptq8_engine_sync(ptq8_engine* e);
/* Reads and clears this engine's device error word, set by bounded waits that ran out
 * (PTQ8_ERR_TIMEOUT; each engine has its own word, so one engine's timeout never
 * aborts or reports through another).  No counterpart in the reference (its kernels
 * have no waits; CUDA errors exit, int8_engine.cuh:109-117). */
int ptq8_engine_check_device_error(ptq8_engine* e);
/* Failure-detection test hook, no counterpart in the reference.  Sets the limit of
 * every bounded device wait of this engine's kernels in clock cycles (0: the default,
 * about 2 s) and, when stall_first_load is nonzero, makes the first operand load of
 * the forward's first tensor-core conv (CTA 0) never arrive, so that the waits on it
 * run out: the forward then reports PTQ8_ERR_TIMEOUT through
 * ptq8_engine_check_device_error / ptq8_engine_sync / ptq8_engine_forward instead of
 * hanging, and the context stays usable.  Drops captured graphs. */
int ptq8_engine_set_wait_test(ptq8_engine* e, long long wait_limit_cycles, int stall_first_load);

/* Parity dumps (replaces forward(..., stop_after_block, mid_out),
 * int8_engine.cuh:429 and locate_block.cpp): what 0 = int8 input codes of conv
 * `index` (NHWC, row pitch shape4[3]; the stem's are its im2col rows), what 1 =
 * the fp32 map fed to the pooling head (NHWC).  shape4 = {N_max, H, W, ld}. */
int ptq8_engine_tensor_info(ptq8_engine* e, int what, int index, int* shape4);
int ptq8_engine_dump(ptq8_engine* e, int what, int index, int n, void* host_dst, size_t bytes);
/* The same for images [n0, n0 + n) of the last forward (the reference oracle runs and
 * dumps a batch chunk by chunk, 06-gpu-int8/cpp/ref_e2e.py:308-329): parity checks of a
 * full-size batch without copying whole multi-GB maps to the host. */
int ptq8_engine_dump_range(ptq8_engine* e, int what, int index, int n0, int n, void* host_dst, size_t bytes);
/* Per-launch timing (CUDA events on the engine stream, `iters` back-to-back
 * launches of each step, not graph-captured) with each step's algorithmic work:
 * ms[i], macs[i], bytes[i], kind[i] (0 stem im2col + GEMM, 1 tensor-core conv,
 * 2 depthwise, 3 maxpool, 4 pooling head) for i < *n_steps (cap entries available).
 * Replaces the reference's PROF_LAYERS per-conv events (int8_engine.cuh:168-176,901-931). */
int ptq8_engine_profile(ptq8_engine* e, int n, int iters, float* ms, double* macs, double* bytes, int* kind,
                        int cap, int* n_steps);
/* Number of kernel launches in one forward (the CUDA graph's kernel nodes). */
int ptq8_engine_n_launches(const ptq8_engine* e);
/* Conv weight bytes the planned engine keeps in device memory, the bytes the same
 * weights take as int8 codes, and how many convs hold W4 codes packed two per byte
 * (W4 convs whose weight slab stays resident in shared memory, and depthwise W4
 * tables).  No counterpart in the reference, whose PTQ2 stores W4 layers as fp32 QDQ
 * values (09-ptq-toolkit/ptq_toolkit/pipeline.py:272-279) and whose engine holds
 * every code as a byte (int8_engine.cuh:211-276). */
int ptq8_engine_weight_bytes(const ptq8_engine* e, size_t* device_bytes, size_t* int8_bytes, int* packed_convs);
/* Human-readable record of what the graph passes did. */
int ptq8_engine_passes_log(const ptq8_engine* e, char* out, size_t cap);

/* ---- one-call interface ----------------------------------------------------
 * The same engine behind five calls, for callers that do not need the steps
 * above.  Status codes only (the reference's forward exits on CUDA errors,
 * int8_engine.cuh:109-117); messages via ptq8_last_error. */

typedef struct ptq8_opts {
    int device;      /* CUDA device ordinal */
    int w_bits;      /* weight bits (8 or 4) when no layer plan is given (Int8Engine::build w_bits) */
    int a_bits;      /* activation bits: 8 */
    int act_mode;    /* PTQ8_ACT_ABSMAX (default, ref_int8.py:69-87) or PTQ8_ACT_MINMAX */
    int passes;      /* PTQ8_PASS_* bits: graph passes on the quantized layers */
    int max_batch;   /* device scratch for this many images; 0: sized by the first forward */
} ptq8_opts;

/* Model::load (ptq_model.h:72) + load_ptqc (:425) + layer plan (mixed_check.py:62-81,
 * per-layer bits 4/8, per_channel only) + Int8Engine::build / set_act_mode /
 * set_calib / alloc_scratch (int8_engine.cuh:132,353,362,807) in one call.  PTQ2
 * and PTQW files are accepted unchanged; plan_json may be NULL.  opts NULL means
 * {device 0, W8, A8, AbsMax, no passes, max_batch 0}.  The engine owns the model.
 * On failure *out is NULL and err holds the message. */
int ptq8_load(const char* model_path, const char* calib_path, const char* plan_json, const ptq8_opts* opts,
              ptq8_engine** out, char* err, size_t errlen);
/* Forward of n images (fp32 NCHW at x_dev) into logits_dev [n][fc_out], both device
 * pointers, asynchronous on `stream` (NULL: the engine's stream).  Replaces
 * Int8Engine::forward (int8_engine.cuh:429) without its host copies. */
int ptq8_forward(ptq8_engine* e, const float* x_dev, int n, float* logits_dev, void* stream);
/* ptq8_forward, then (synchronously) the int8 input codes of every conv, handed to
 * dump(user, conv, codes, n, h, w, ld) as a host array [n][h][w][ld] (the stem's
 * are its im2col rows) -- the parity hook that replaces forward(...,
 * stop_after_block, mid_out) and locate_block.cpp. */
typedef void (*ptq8_dump_fn)(void* user, int conv, const int8_t* codes, int n, int h, int w, int ld);
int ptq8_forward_debug(ptq8_engine* e, const float* x_dev, int n, float* logits_dev, void* stream,
                       ptq8_dump_fn dump, void* user);
/* Capture (and cache) the CUDA graph of a forward at batch n ahead of the first
 * forward (the reference launches kernel by kernel with no graph). */
int ptq8_capture_graph(ptq8_engine* e, int n);
/* Destroy an engine and, when it came from ptq8_load, its model. */
void ptq8_destroy(ptq8_engine* e);
const char* ptq8_last_error(const ptq8_engine* e);

#ifdef __cplusplus
}
#endif

#endif /* PTQ8_H */
