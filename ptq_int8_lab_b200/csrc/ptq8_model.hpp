// Calibrated-model interface of the engine: PTQW / PTQ2 weights+topology,
// PTQC activation ranges, per-tensor activation scale and per-channel weight
// quantization.  CPU-only (no CUDA types), so it is unit-tested without a GPU.
//
// File formats (little endian), as written by the reference toolchain:
//   PTQW  06-gpu-int8/cpp/export_weights.py:12-21, read by ptq_model.h:257-346
//         "PTQW", i32 n_conv, n_block, stem_pool;
//         per conv 9 x i32 (cout cin kh kw sh sw ph pw relu) + f32 weight + f32 bias;
//         per block 4 x i32 (c1 c2 ds stride); i32 fc_in fc_out + f32 weight + f32 bias.
//   PTQ2  09-ptq-toolkit/ptq_toolkit/export/topoblocks.py:17-35,247-267, read by
//         06-gpu-int8/cpp/ptq2_reader.h:112-270
//         "PTQ2", i32 n_conv, n_block, stem_pool, ncp;
//         per conv 10 x i32 (... relu groups) + weights + bias;
//         per block (ncp + 3) x i32 (convs..., -1 padded, ds, stride, residual); fc.
//   PTQC  09-ptq-toolkit/ptq_toolkit/export/ptqc.py:1-20, read by ptq_model.h:425-503
//         "PTQC", i32 n, n x (f32 lo, f32 hi); size exactly 8 + 8n.
//   PTQ8  this engine's native package (no reference counterpart: the reference's PTQ2
//         stores every layer, W4 included, as fp32 QDQ values, pipeline.py:272-279):
//         "PTQ8", i32 version (1), n_conv, n_block, stem_pool, ncp;
//         per conv 10 x i32 as PTQ2, i32 bits (8 or 4), f32 w_scale[cout], f32 bias[cout],
//         codes: bits 8 -> int8 [cout][K]; bits 4 -> [cout][ceil(K/2)] bytes, code k of a
//         row in the low nibble of byte k/2 for even k, the high nibble for odd k
//         (K = cin * kh * kw in (c, i, j) order, the per-channel codes of
//         ptq_quant.h:72-110); per block (ncp + 3) x i32 as PTQ2; fc as PTQ2.
//
// Error behaviour mirrors the reference loaders: every failure returns false
// with a message, nothing exits, truncated files and trailing bytes are
// rejected, topology is validated (ptq_model.h:104-203).
#pragma once

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace ptq8 {

struct ConvSpec {
    int cout = 0, cin = 0, kh = 0, kw = 0;   // cin = input channels per group
    int sh = 1, sw = 1, ph = 0, pw = 0;
    int relu = 0;                             // 0 none, 1 ReLU, 2 ReLU6
    int groups = 1;
    std::vector<float> weight;                // [cout][cin][kh][kw] (empty when qbits > 0)
    std::vector<float> bias;                  // [cout]
    // PTQ8: the per-channel codes and f32 scales as stored (qbits 8 or 4; 0 for fp32 weights)
    int qbits = 0;
    std::vector<int8_t> codes;                // [cout][cin * kh * kw], one code per byte
    std::vector<float> wscale;                // [cout]
    int in_channels() const { return cin * groups; }
    bool depthwise() const { return cin == 1 && groups == cout && groups > 1; }
};

struct BlockSpec {
    std::vector<int> convs;   // execution order, -1 padding only at the tail
    int ds = -1;              // identity-branch conv, -1 = direct
    int stride = 1;
    int residual = 1;         // 0 none, 1 add then ReLU, 2 add only
};

struct Model {
    std::vector<ConvSpec> convs;
    std::vector<BlockSpec> blocks;
    int stem_pool = 0;
    int fc_in = 0, fc_out = 0;
    std::vector<float> fc_w, fc_b;   // [fc_out][fc_in], [fc_out]
    std::string magic;               // "PTQW", "PTQ2" or "PTQ8"

    // Model::load (ptq_model.h:72-91): dispatch on magic, strict parse, validate.
    bool load(const std::string& path, std::string* err);
    // Topology check (ptq_model.h:104-203) for a given input spatial size.
    bool validate(std::string* err, int input_h = 32, int input_w = 32) const;
};

// load_ptqc (ptq_model.h:425-503): 8+8n bytes, n == n_expected, finite, lo <= hi.
bool load_ptqc(const std::string& path, size_t n_expected,
               std::vector<std::pair<float, float>>* out, std::string* err);

// Activation scale (ptq_quant.h:195-214 / ref_int8.py:69-87), kept in float64:
// the reference oracle divides by the float64 scale.
enum ActMode { ACT_ABSMAX = 0, ACT_MINMAX = 1 };
double act_scale_from_range(float lo, float hi, int bits, int mode);

// Per-output-channel symmetric weight codes (ptq_quant.h:72-110 /
// ref_int8.py:146-160): scale64 = max(amax/qmax, 1e-8), code =
// clip(round_half_away(w/scale64), -(qmax+1), qmax), scale stored as f32.
void quantize_weight_per_channel(const float* w, int cout, int k, int bits,
                                 int8_t* codes, float* scale32);

int conv_out_dim(int in, int k, int s, int p);

// Per-conv weight bits from a layer-plan JSON (the `layers` list of the
// ptq-layer-plan/v1 schema, mixed_check.py:62-81 / mixed.py:179): exactly
// n_conv entries in conv definition order, bits 4 or 8, scheme per_channel.
bool load_layer_plan(const std::string& path, size_t n_conv, std::vector<int>* bits, std::string* err);

}  // namespace ptq8
