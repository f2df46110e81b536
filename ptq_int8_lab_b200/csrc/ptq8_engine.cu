// Int8 engine: topology interpreter, device buffers, TMA descriptors, CUDA
// graph replay, and the extern "C" boundary declared in include/ptq8.h.
//
// Execution model (mirrors Int8Engine::forward, 06-gpu-int8/cpp/int8_engine.cuh:429-645,
// and the topology semantics of 09-.../export/topoblocks.py:181-220):
//   stem conv [-> maxpool] -> blocks (ds conv first, then the block's convs;
//   the residual add + post activation run in the last conv's epilogue) ->
//   global average pool + FC.
// Every intermediate is a separate device buffer (no aliasing), so any conv's
// input codes can be dumped after a forward for bit-exact parity checks.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include "ptq8_kernels.cuh"
#include "ptq8_model.hpp"
#include "ptq8.h"

using namespace ptq8;

namespace {


std::string strf(const char* f, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, f);
    std::vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return buf;
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Normalisation constants of 8-bit CIFAR-10 pixels, computed in float32 as the
// reference's input paths compute them: m = mean * 255; kNormDiv: d = std * 255
// (ref_e2e.py:272-274, numpy float32); kNormMul: d = 1 / (std * 255)
// (main.cpp:25-26,257-258).
U8Norm make_norm(int mode, const float* mean, const float* sd, int c) {
    U8Norm nm{};
    nm.mode = mode;
    for (int k = 0; k < c; ++k) {
        const volatile float m = mean[k] * 255.0f;   // each float32 operation rounded on its own
        const volatile float d = sd[k] * 255.0f;
        nm.m[k] = m;
        nm.d[k] = mode == kNormMul ? 1.0f / d : d;
    }
    return nm;
}

U8Norm cifar_norm(int mode) {
    static const float kMean[3] = {0.4914f, 0.4822f, 0.4465f}, kStd[3] = {0.2470f, 0.2435f, 0.2616f};
    return make_norm(mode, kMean, kStd, 3);
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

CUtensorMapSwizzle swizzle_for(int cb) {
    return cb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (cb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// An fp32 activation of the network and the int8 code tensors made from it.
struct Value {
    int h = 0, w = 0, c = 0;   // per-image NHWC shape
    bool need_f32 = false;
    std::vector<double> scales;  // distinct consumer scales, in first-use order
    int ldq = 0;                 // code row pitch (c rounded up to 32)
    float* f32 = nullptr;
    std::vector<int8_t*> codes;  // one per scale
    std::vector<char> sub2;      // per scale: codes kept only at even (h, w), half-size bordered map
    int sub_h() const { return (h + 1) / 2; }
    int sub_w() const { return (w + 1) / 2; }
    bool is_sub(int k) const { return k >= 0 && k < (int)sub2.size() && sub2[k]; }
    int code_index(double s) const {
        for (size_t i = 0; i < scales.size(); ++i)
            if (scales[i] == s) return (int)i;
        return -1;
    }
};

enum LaunchKind { K_STEM_IM2COL = 0, K_TC = 1, K_DW = 2, K_MAXPOOL = 3 };

struct Step {
    int kind = K_TC;
    int conv = -1;        // model conv index (or -1 for maxpool)
    int in_val = -1;      // value read (codes at conv scale; fp32 for maxpool)
    int out_val = -1;     // value produced
    int res_val = -1;     // residual value (fp32), -1 none
    int post = 0;         // 0 none, 1 add + relu, 2 add
    int act = 0;
    // geometry
    int ih = 0, iw = 0, ic = 0, oh = 0, ow = 0, oc = 0;
    int kh = 1, kw = 1, sh = 1, sw = 1, ph = 0, pw = 0;
    int cb = 32, bn = 16, n_ntiles = 1, ktot = 0, kpad = 0;
    int stages = 4, b_resident = 0, n_kchunks = 1;
    int mode = 0;          // 0 per-tap tile loads, 1 halo block + shifted views (see conv_tc_kernel)
    int blk_rows = 0;      // mode 1: bordered rows per block
    int a_stage = 0;       // bytes per A pipeline stage
    size_t smem = 0;
    int grid_x = 1;
    void* kfn = nullptr;   // conv_tc_kernel specialization
    int TW = 1, TH = 1, TN = 1;
    double s_in = 1.0;
    // device parameters
    int8_t* d_w = nullptr;
    uint8_t* d_w4 = nullptr;    // W4 codes two per byte (resident-slab tensor-core convs), else null
    bool w_packed = false;      // d_w4 (tensor-core) / a packed d_dwt table (depthwise) holds the weights
    size_t w_dev_bytes = 0;     // bytes of this step's weights in device memory
    float* d_factor = nullptr;
    float* d_bias = nullptr;
    std::vector<float> h_factor, h_bias;   // host copies (tensor-core convs take them as kernel parameters)
    int8_t* d_im2col = nullptr;   // stem rows, bordered [N][OH+2][OW+2][kpad]
    CUtensorMap map_a{}, map_b{};
    // aux GEMM: this conv recomputes its residual (the stem's output) from the
    // stem's im2col rows instead of reading a stored fp32 map
    int aux_src = -1;      // step index of the recomputed conv (stem or fused downsample), -1 none
    int aux_kb = 32;       // K bytes of that GEMM
    bool fused = false;    // a downsample computed inside its block's last conv: never launched
    int aux_off = 0;       // byte offset of the aux tile inside an A stage
    int acc_cols = 0;      // TMEM columns per accumulator buffer (main + aux)
    bool fast = false;     // conv_tc_kernel with the compile-time N tile epilogue (epilogue_fast)
    CUtensorMap map_xa{}, map_xb{};
    // depthwise 3x3 / pad 1 / stride 1-2 (dw3x3_kernel): dp4a weight table, 3 uint4 per
    // word of 4 channels; consumer threads (a multiple of 32 and of the word count), strip
    // length T, unit shape (R output rows of one image, or k whole images), staged rows per
    // image, stage bytes and count, CTAs of the persistent grid, kernel specialization
    uint4* d_dwt = nullptr;
    // |acc| <= 128 * max_c sum_k |w[c][k]| < 2^22: accumulators convert to float without a range check
    bool acc_small = false;
    int dw_cons = 0, dw_T = 1, dw_R = 1, dw_kimg = 1, dw_rows = 0, dw_stage = 0, dw_stages = 2, dw_ctas = 1;
    void* dw_kfn = nullptr;
};

struct ConvQ {   // quantized conv after graph passes
    ConvSpec spec;              // geometry (weight field unused)
    int bits = 8;
    std::vector<int8_t> codes;  // [cout][cin*kh*kw] in (c,i,j) order
    std::vector<float> wscale;  // [cout]
    std::vector<float> bias;
    // positional decomposition: output channel c' = pos*cout_orig + c (NHWC == D2S DCR)
    int view_oh = 0, view_ow = 0;   // >0 when the conv runs as a 1x1-output GEMM
    // generalised positional decomposition: per-position sub-convs (each output position of
    // TN images is one M tile that multiplies only its in-bounds taps)
    bool pos_tiles = false;
};

}  // namespace

struct ptq8_model {
    Model m;
};

struct ptq8_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    std::string err;
    const Model* model = nullptr;   // caller keeps the model alive (int8_engine.cuh:134)
    ptq8_model* owned_model = nullptr;   // set by ptq8_load: freed with the engine
    int w_bits = 8, a_bits = 8, act_mode = ACT_ABSMAX, passes = 0;
    std::vector<int> layer_bits;
    std::vector<ConvQ> q;
    std::vector<std::pair<float, float>> ranges;
    std::vector<double> scale;     // per conv input scale (double)
    bool built = false, calibrated = false, planned = false;
    int in_c = 3, in_h = 32, in_w = 32;
    int max_batch = 0;
    int max_ctas = 0;   // cap on the persistent grid of each tensor-core conv (0: all SMs)
    // plan
    std::vector<Value> vals;
    std::vector<Step> steps;
    int final_val = -1;
    std::vector<int> conv_step;    // conv index -> step index
    float* d_input = nullptr;      // fp32 NCHW [max_batch][3][32][32]
    // pipelined host-buffer forward (ptq8_engine_forward_async): second input slot,
    // copy stream, per-slot events, next slot; graphs are keyed by batch * 2 + slot
    float* d_input2 = nullptr;
    const float* cur_input = nullptr;   // the input the stem reads while a forward is enqueued
    // 8-bit pixel input (ptq8_engine_forward_u8*): two lazily allocated slots [max_batch][c*h*w],
    // the normalisation the stem applies, and the slot a forward being enqueued reads
    uint8_t* d_input_u8[2] = {nullptr, nullptr};
    const uint8_t* cur_input_u8 = nullptr;
    U8Norm u8_norm = cifar_norm(kNormDiv);
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_staged[2] = {nullptr, nullptr}, ev_free[2] = {nullptr, nullptr};
    int async_slot = 0;
    float* d_logits = nullptr;
    float* d_fc_w = nullptr;
    float* d_fc_b = nullptr;
    // device error word of this engine's kernels (bounded waits that ran out), the wait
    // limit they get, and the failure-detection test switch (ptq8_engine_set_wait_test)
    int* d_err = nullptr;
    long long wait_limit = kWaitLimitCycles;
    int stall_first_load = 0;
    std::vector<void*> allocs;
    std::map<int, cudaGraphExec_t> graphs;
    std::vector<std::string> passes_log;

    ~ptq8_engine() { release(); }

    void release() {
        if (copy_stream) cudaStreamSynchronize(copy_stream);
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
        for (void* p : allocs) cudaFree(p);
        allocs.clear();
        d_input2 = nullptr;
        for (int k = 0; k < 2; ++k) {
            if (ev_staged[k]) cudaEventDestroy(ev_staged[k]);
            if (ev_free[k]) cudaEventDestroy(ev_free[k]);
            ev_staged[k] = ev_free[k] = nullptr;
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
        copy_stream = nullptr;
        if (own_stream && stream) cudaStreamDestroy(stream);
        stream = nullptr;
        own_stream = false;
    }

    int fail(const std::string& m, int code = PTQ8_ERR_INVALID) {
        err = m;
        return code;
    }

    bool cuda_ok(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        err = strf("%s: %s", what, cudaGetErrorString(e));
        return false;
    }

    template <class T>
    bool dalloc(T** p, size_t bytes, const char* what) {
        void* v = nullptr;
        if (!cuda_ok(cudaMalloc(&v, bytes ? bytes : 16), what)) return false;
        allocs.push_back(v);
        *p = reinterpret_cast<T*>(v);
        return true;
    }
};

namespace {

// ------------------------------------------------------------------ graph passes

// Center tap (07-tensorrt-deploy/scripts/push_optimize_onnx.py:36-93): a kxk conv
// (k odd, stride 1, pad (k-1)/2) whose input and output maps are 1x1 only ever
// multiplies the center tap by real data; the others see padding code 0.  The
// rewrite keeps the int8 codes of the center tap and the per-channel scales of
// the full kernel, so the int32 accumulators are unchanged.
bool center_tap(ConvQ& cq, int ih, int iw, std::string* note) {
    ConvSpec& c = cq.spec;
    if (ih != 1 || iw != 1 || c.kh != c.kw || c.kh % 2 == 0 || c.kh == 1) return false;
    if (c.sh != 1 || c.sw != 1 || c.ph != c.kh / 2 || c.pw != c.kw / 2 || c.groups != 1) return false;
    const int k = c.kh, ctr = k / 2, cin = c.cin;
    std::vector<int8_t> nc((size_t)c.cout * cin);
    for (int o = 0; o < c.cout; ++o)
        for (int ci = 0; ci < cin; ++ci)
            nc[(size_t)o * cin + ci] = cq.codes[(((size_t)o * cin + ci) * k + ctr) * k + ctr];
    cq.codes.swap(nc);
    c.kh = c.kw = 1;
    c.ph = c.pw = 0;
    *note = strf("center-tap %dx%d -> 1x1", k, k);
    return true;
}

// One spatial dimension of the positional decomposition
// (07-tensorrt-deploy/scripts/push_decompose.py:50-80): per output position the
// valid kernel slice; uniform when every position reads the whole input with
// the same number of taps.
bool uniform_dim(int H, int k, int p, int s, int* OH, int* t, std::vector<int>* los) {
    *OH = (H + 2 * p - k) / s + 1;
    los->clear();
    int tt = -1;
    for (int i = 0; i < *OH; ++i) {
        const int lo = std::max(0, p - s * i);
        const int hi = std::min(k - 1, H - 1 + p - s * i);
        if (lo > hi) return false;
        const int r_lo = s * i - p + lo, r_hi = s * i - p + hi;
        if (r_lo != 0 || r_hi != H - 1) return false;
        if (tt < 0) tt = hi - lo + 1;
        if (hi - lo + 1 != tt) return false;
        los->push_back(lo);
    }
    *t = tt;
    return true;
}

// Positional decomposition (push_decompose.py:99-202): a conv whose input map is
// no larger than its kernel becomes one th x tw conv with OH*OW*cout outputs
// (position-major weight blocks, tiled bias) followed by DepthToSpace(DCR).
// The epilogue applies the DCR rearrangement as it writes: output channel
// (i*OW+j)*cout + c of image n goes to element (n, i, j, c) of the OH x OW map
// (code_ptr for codes, f32_at for the fp32 map).  Codes and scales are sliced
// from the quantized kernel, so the accumulators are unchanged.
bool decompose(ConvQ& cq, int H, int W, std::string* note) {
    ConvSpec& c = cq.spec;
    if (c.groups != 1 || c.kh != c.kw || c.kh % 2 == 0) return false;
    const int k = c.kh, p = (k - 1) / 2;
    if (c.ph != p || c.pw != p) return false;
    if (H > k || W > k) return false;
    int OH, OW, th, tw;
    std::vector<int> lh, lw;
    if (!uniform_dim(H, k, p, c.sh, &OH, &th, &lh) || !uniform_dim(W, k, p, c.sw, &OW, &tw, &lw)) return false;
    if (th == k && tw == k && p == 0) return false;
    if (OH > 1 && OH != OW) return false;
    // NHWC identity of the DCR rearrangement needs the code rows unpadded
    if ((OH > 1 || OW > 1) && c.cout % 32 != 0) return false;
    const int cout = c.cout, cin = c.cin;
    const int ncout = OH * OW * cout;
    std::vector<int8_t> nc((size_t)ncout * cin * th * tw);
    std::vector<float> ns((size_t)ncout), nb((size_t)ncout);
    for (int i = 0; i < OH; ++i)
        for (int j = 0; j < OW; ++j) {
            const int blk = (i * OW + j) * cout;
            for (int o = 0; o < cout; ++o) {
                ns[blk + o] = cq.wscale[o];
                nb[blk + o] = cq.bias[o];
                for (int ci = 0; ci < cin; ++ci)
                    for (int a = 0; a < th; ++a)
                        for (int b = 0; b < tw; ++b)
                            nc[(((size_t)(blk + o) * cin + ci) * th + a) * tw + b] =
                                cq.codes[(((size_t)o * cin + ci) * k + lh[i] + a) * k + lw[j] + b];
            }
        }
    *note = strf("decompose %dx%d s%d on %dx%d -> %dx%d conv, %d outputs%s", k, k, c.sh, H, W, th, tw, ncout,
                 (OH > 1 || OW > 1) ? strf(" + DepthToSpace(%d)", OH).c_str() : "");
    cq.codes.swap(nc);
    cq.wscale.swap(ns);
    cq.bias.swap(nb);
    cq.view_oh = OH;
    cq.view_ow = OW;
    c.cout = ncout;
    c.kh = th;
    c.kw = tw;
    c.sh = c.sw = 1;
    c.ph = c.pw = 0;
    return true;
}

// Generalised positional decomposition: the per-position sub-convs of a conv whose
// output positions read different kernel slices (07-tensorrt-deploy/scripts/
// push_decompose.py:50-80 computes the slice per position; its decompose() needs every
// position to read the whole input with the same slice, which the CIFAR-stem ResNet-18's
// 8x8 and 4x4 maps never do).  Output position (i, j) is the GEMM of the images' codes
// under kernel rows [lo_h(i), hi_h(i)] and columns [lo_w(j), hi_w(j)] -- the taps that
// read inside the input -- with the same codes' weights: the dropped taps multiply padding
// code 0, so every int32 accumulator is unchanged.  The engine runs each position as its
// own M tiles (TN images at one position; mode 0) and skips the dropped taps' K chunks.
// Applied to output maps of at most 64 positions where the dropped taps are at least 5 %
// of the conv's MACs.
bool positional(ConvQ& cq, int H, int W, std::string* note) {
    const ConvSpec& c = cq.spec;
    if (c.groups != 1 || c.kh == 1 || c.kw == 1 || cq.view_oh > 0) return false;
    const int OH = (H + 2 * c.ph - c.kh) / c.sh + 1, OW = (W + 2 * c.pw - c.kw) / c.sw + 1;
    // larger maps keep their row-block tiles (the halo-block pipeline of stride-1 convs)
    if (OH < 1 || OW < 1 || OH * OW > 64) return false;
    long long full = 0, kept = 0;
    int classes_h = 0, classes_w = 0, prev_h = -1, prev_w = -1;
    for (int i = 0; i < OH; ++i) {
        const int lo = std::max(0, c.ph - c.sh * i), hi = std::min(c.kh - 1, H - 1 + c.ph - c.sh * i);
        if (lo > hi) return false;
        if (lo * 64 + hi != prev_h) { ++classes_h; prev_h = lo * 64 + hi; }
        for (int j = 0; j < OW; ++j) {
            const int lw = std::max(0, c.pw - c.sw * j), hw = std::min(c.kw - 1, W - 1 + c.pw - c.sw * j);
            if (lw > hw) return false;
            if (i == 0 && lw * 64 + hw != prev_w) { ++classes_w; prev_w = lw * 64 + hw; }
            full += (long long)c.kh * c.kw;
            kept += (long long)(hi - lo + 1) * (hw - lw + 1);
        }
    }
    if ((full - kept) * 20 < full) return false;   // under 5 % of the MACs read padding
    cq.pos_tiles = true;
    const long long macs = (long long)c.cout * c.cin;
    *note = strf("positional %dx%d s%d on %dx%d -> %d position classes (%dx%d), MACs %lld -> %lld per image",
                 c.kh, c.kw, c.sh, H, W, classes_h * classes_w, classes_h, classes_w, full * macs, kept * macs);
    return true;
}

// ------------------------------------------------------------------ planning

int new_value(ptq8_engine* e, int h, int w, int c) {
    Value v;
    v.h = h;
    v.w = w;
    v.c = c;
    v.ldq = round_up(c, 32);
    e->vals.push_back(v);
    return (int)e->vals.size() - 1;
}

void need_codes(ptq8_engine* e, int val, double s) {
    Value& v = e->vals[val];
    if (v.code_index(s) < 0) v.scales.push_back(s);
}

void tile_shape(int N, int OH, int OW, int* TW, int* TH, int* TN) {
    if (OW >= 128) {
        *TW = 128; *TH = 1; *TN = 1;
        return;
    }
    *TW = OW;
    *TH = std::max(1, std::min(OH, 128 / OW));
    *TN = std::max(1, std::min(128 / (OW * *TH), 256));
    (void)N;
}

constexpr size_t kSmemBudget = 225 * 1024;

int choose_cb(int cpad) { return cpad % 128 == 0 ? 128 : (cpad % 64 == 0 ? 64 : 32); }

// N tile: the whole Cout when it fits one MMA (N <= 256, multiple of 16);
// otherwise equal tiles rounded up to 32 channels, so that every tile's first
// channel keeps the 32-byte alignment of the epilogue's vector stores.
void choose_bn(int cout, int* bn, int* ntiles) {
    if (cout <= 256) {
        *ntiles = 1;
        *bn = round_up(cout, 16);
        return;
    }
    int nt = (cout + 255) / 256;
    int b = round_up((cout + nt - 1) / nt, 32);
    nt = (cout + b - 1) / b;
    *ntiles = nt;
    *bn = b;
}

// Whether the downsample `ds` (1x1 stride 2, no activation) of a block can run
// inside the block's last conv `ci` as its aux GEMM: `ci` is a 3x3 stride-1
// "same" conv on the downsample's output map in halo-block mode, N tile = all
// channels (<= 128, so main + aux accumulators fit twice in TMEM), and the
// block input is produced by a tensor-core conv (its epilogue writes the
// subsampled codes the aux GEMM reads).
// Depthwise convs that dw3x3_kernel runs: 3x3, padding 1, equal strides of 1 or 2,
// codes out only (no residual, fp32 map or subsampled output), and a 4-channel word
// count G4 with lcm(32, G4) <= 640 (the consumer threads are a multiple of both).
bool dw3x3_eligible(const ptq8_engine* e, const Step& st) {
    const int G4 = (st.oc + 3) / 4;
    const Value& out = e->vals[st.out_val];
    bool sub = false;
    for (size_t k = 0; k < out.scales.size(); ++k) sub = sub || out.is_sub((int)k);
    return st.kh == 3 && st.kw == 3 && st.ph == 1 && st.pw == 1 && st.sh == st.sw && (st.sh == 1 || st.sh == 2) &&
           st.res_val < 0 && !out.need_f32 && !sub && st.act >= 0 && st.act <= 2 && !out.scales.empty() &&
           out.scales.size() <= 2 && 32 / std::gcd(32, G4) * G4 <= kDwMaxConsumers;
}

// dw3x3_kernel specializations [T = 1, 2, 4][stride 1, 2][act 0, 1, 2]
using DwKernel = void (*)(const int8_t*, const uint4*, const DwGeom, const EpiParams);
template <int T, int S>
constexpr DwKernel dw_k(int act) {
    return act == 0 ? dw3x3_kernel<T, S, 0> : act == 1 ? dw3x3_kernel<T, S, 1> : dw3x3_kernel<T, S, 2>;
}
DwKernel dw_kernel_for(int T, int S, int act) {
    if (T == 4) return S == 1 ? dw_k<4, 1>(act) : dw_k<4, 2>(act);
    if (T == 2) return S == 1 ? dw_k<2, 1>(act) : dw_k<2, 2>(act);
    return S == 1 ? dw_k<1, 1>(act) : dw_k<1, 2>(act);
}

// Strip length, unit shape, consumer count and pipeline depth of a dw3x3_kernel
// launch (see the kernel).  Among consumer counts that are multiples of
// lcm(32, G4) in [256, 640] and units whose staged bytes fit kDwStageMax, take the
// best product of thread use (strips x words per unit over whole passes of the
// consumers) and staged-row use (output rows x stride over staged rows); ties go to
// more consumers, then to the larger unit.
constexpr int kDwStageMax = 100 * 1024;
constexpr int kDwSmemLimit = 210 * 1024;   // dynamic shared memory of any plan

bool plan_dw3x3(const ptq8_engine* e, Step& st, int max_batch) {
    const Value& vin = e->vals[st.in_val];
    const int G4 = (st.oc + 3) / 4, S = st.sh;
    st.dw_T = st.ow % 4 == 0 ? 4 : st.ow % 2 == 0 ? 2 : 1;
    const long strips = st.ow / st.dw_T;
    const long row = (long)(st.iw + 2) * vin.ldq;
    const int l = 32 / std::gcd(32, G4) * G4;
    std::vector<int> cons;
    for (int b = l; b <= kDwMaxConsumers; b += l)
        if (b >= 256 || b + l > kDwMaxConsumers) cons.push_back(b);
    double best = -1.0;
    auto consider = [&](int R, int k, int rows) {
        const long bytes = (long)k * rows * row;
        if (bytes > kDwStageMax) return;
        const int stage = (int)((bytes + 127) / 128 * 128);
        const int stages = std::min(kDwMaxStages, kDwSmemLimit / stage);
        if (stages < 2) return;
        const long items = (long)k * R * strips * G4;
        const double rows_use = (double)(S * R) / rows;
        for (int b : cons) {
            const long passes = (items + b - 1) / b;
            const double score = (double)items / (double)(passes * b) * rows_use + 1e-6 * b + 1e-9 * (double)items;
            if (score > best) {
                best = score;
                st.dw_cons = b;
                st.dw_R = R;
                st.dw_kimg = k;
                st.dw_rows = rows;
                st.dw_stage = stage;
                st.dw_stages = stages;
            }
        }
    };
    for (int R = 1; R <= st.oh; ++R)
        if (st.oh % R == 0) consider(R, 1, S * (R - 1) + 3);
    for (int k = 2; k <= std::max(2, max_batch) && (long)k * (st.ih + 2) * row <= kDwStageMax; ++k)
        consider(st.oh, k, st.ih + 2);
    st.dw_kfn = (void*)dw_kernel_for(st.dw_T, S, st.act);
    return best > 0.0;
}

bool ds_fusable(const ptq8_engine* e, int ds, int ci, int in_val) {
    const ConvSpec& d = e->q[ds].spec;
    const ConvSpec& c = e->q[ci].spec;
    if (e->q[ds].view_oh > 0 || d.groups != 1 || d.kh != 1 || d.kw != 1 || d.sh != 2 || d.sw != 2 || d.ph != 0 ||
        d.pw != 0 || d.relu != 0)
        return false;
    const int kb = round_up(d.cin, 32);
    if (kb > 128) return false;
    if (e->q[ci].view_oh > 0 || c.groups != 1 || c.kh != 3 || c.kw != 3 || c.sh != 1 || c.sw != 1 || c.ph != 1 ||
        c.pw != 1)
        return false;
    if (c.cout != d.cout || c.cout > 128 || c.cout % 16 != 0 || round_up(c.cin, 32) % 64 != 0) return false;
    const Value& x = e->vals[in_val];
    const int oh = (x.h + 1) / 2, ow = (x.w + 1) / 2;
    if (oh * ow < 64 || 128 + 2 * (ow + 2) + 2 > 256) return false;
    // halo-block pipeline with resident weights and two stages must fit in shared memory
    const int cpad = round_up(c.cin, 32), cb = choose_cb(cpad), bn = round_up(c.cout, 16);
    const size_t b_res = (size_t)9 * (cpad / cb) * round_up(bn * cb, 1024);
    const size_t stage = (size_t)round_up((128 + 2 * (ow + 2) + 2) * cb, 1024) + 128 * kb;
    if (1024 + 2 * stage + b_res + (size_t)round_up(bn * kb, 1024) > kSmemBudget) return false;
    for (const Step& st : e->steps)
        if (st.out_val == in_val) return st.kind == K_TC || st.kind == K_STEM_IM2COL;
    return false;
}

// Whether the block conv `ci`, whose residual is the stem's output, can recompute
// that residual from the stem's im2col rows (one K = 32 GEMM in its own kernel)
// instead of reading it as a stored fp32 map: a 3x3 stride-1 "same" conv on the
// stem's map (halo-block mode), N tile = all channels, same channel count.
bool stem_identity_fusable(const ptq8_engine* e, int ci) {
    const Model& m = *e->model;
    if (m.stem_pool) return false;
    const ConvSpec& st = e->q[0].spec;
    const ConvSpec& c = e->q[ci].spec;
    if (st.cin * st.kh * st.kw > 32 || st.groups != 1) return false;
    if (e->q[ci].view_oh > 0 || c.groups != 1 || c.kh != 3 || c.kw != 3 || c.sh != 1 || c.sw != 1 || c.ph != 1 ||
        c.pw != 1)
        return false;
    if (c.cout != st.cout || c.cout > 128 || c.cout % 16 != 0 || round_up(c.cin, 32) % 64 != 0) return false;
    const int oh = conv_out_dim(e->in_h, st.kh, st.sh, st.ph), ow = conv_out_dim(e->in_w, st.kw, st.sw, st.pw);
    return oh * ow >= 64 && 128 + 2 * (ow + 2) + 2 <= 256;
}

int plan(ptq8_engine* e) {
    const Model& m = *e->model;
    e->vals.clear();
    e->steps.clear();
    e->conv_step.assign(m.convs.size(), -1);

    // --- shapes of every conv input, computed along the topology
    std::vector<int> in_h(m.convs.size(), 0), in_w(m.convs.size(), 0);
    auto add_conv = [&](int ci, int in_val, int* out_val, int res_val, int post) -> int {
        const Value& vin = e->vals[in_val];
        ConvQ& cq = e->q[ci];
        const ConvSpec& c = cq.spec;
        Step st;
        st.conv = ci;
        st.in_val = in_val;
        st.ih = vin.h;
        st.iw = vin.w;
        st.ic = c.in_channels();
        st.kh = c.kh; st.kw = c.kw; st.sh = c.sh; st.sw = c.sw; st.ph = c.ph; st.pw = c.pw;
        st.act = c.relu;
        st.s_in = e->scale[ci];
        int oh = conv_out_dim(vin.h, c.kh, c.sh, c.ph), ow = conv_out_dim(vin.w, c.kw, c.sw, c.pw);
        int oc = c.cout;
        if (cq.view_oh > 0) {   // decomposed conv: outputs as (view_oh, view_ow, cout/(view_oh*view_ow))
            oc = c.cout / (cq.view_oh * cq.view_ow);
            st.oh = 1; st.ow = 1;
        } else {
            st.oh = oh; st.ow = ow;
        }
        const int vh = cq.view_oh > 0 ? cq.view_oh : oh, vw = cq.view_ow > 0 ? cq.view_ow : ow;
        st.oc = c.cout;
        *out_val = new_value(e, vh, vw, oc);
        st.out_val = *out_val;
        st.res_val = res_val;
        st.post = post;
        if (c.depthwise()) {
            st.kind = K_DW;
        } else if (c.groups != 1) {
            return e->fail(strf("conv[%d]: grouped conv with groups=%d (not depthwise) is not supported", ci, c.groups));
        } else {
            st.kind = K_TC;
        }
        if (e->vals[in_val].f32 == nullptr && in_val == 0 && ci == 0) st.kind = K_STEM_IM2COL;
        if (st.kind != K_STEM_IM2COL) need_codes(e, in_val, e->scale[ci]);
        e->conv_step[ci] = (int)e->steps.size();
        e->steps.push_back(st);
        return PTQ8_OK;
    };

    // value 0: network input (fp32 NCHW, read by the stem im2col kernel)
    new_value(e, e->in_h, e->in_w, e->in_c);
    int cur = -1;
    int rc = add_conv(0, 0, &cur, -1, 0);
    if (rc) return rc;
    const int stem_val = cur, stem_step = (int)e->steps.size() - 1;
    if (m.stem_pool) {
        Value& v0 = e->vals[cur];
        v0.need_f32 = true;
        const int ph = (v0.h + 2 - 3) / 2 + 1, pw = (v0.w + 2 - 3) / 2 + 1;
        const int pv = new_value(e, ph, pw, v0.c);
        Step st;
        st.kind = K_MAXPOOL;
        st.in_val = cur;
        st.out_val = pv;
        st.ih = e->vals[cur].h; st.iw = e->vals[cur].w; st.ic = e->vals[cur].c;
        st.oh = ph; st.ow = pw; st.oc = e->vals[cur].c;
        e->steps.push_back(st);
        cur = pv;
    }
    for (size_t bi = 0; bi < m.blocks.size(); ++bi) {
        const BlockSpec& b = m.blocks[bi];
        std::vector<int> cs;
        for (int ci : b.convs)
            if (ci >= 0) cs.push_back(ci);
        int ident = -1;
        bool fuse = false;
        int ds_step = -1;
        if (b.residual != 0) {
            if (b.ds >= 0) {
                int dv;
                rc = add_conv(b.ds, cur, &dv, -1, 0);
                if (rc) return rc;
                ident = dv;
                if (!cs.empty() && ds_fusable(e, b.ds, cs.back(), cur)) ds_step = (int)e->steps.size() - 1;
            } else {
                ident = cur;
            }
            fuse = ident == stem_val && !cs.empty() && stem_identity_fusable(e, cs.back());
            if (!fuse && ds_step < 0) e->vals[ident].need_f32 = true;
        }
        int t = cur;
        for (size_t k = 0; k < cs.size(); ++k) {
            const bool last = k + 1 == cs.size();
            int ov;
            rc = add_conv(cs[k], t, &ov, last && b.residual ? ident : -1, last ? b.residual : 0);
            if (rc) return rc;
            if (last && fuse) {
                e->steps.back().aux_src = stem_step;
                e->steps.back().aux_kb = 32;
            }
            if (last && ds_step >= 0) {
                e->steps.back().aux_src = ds_step;
                e->steps.back().aux_kb = round_up(e->q[b.ds].spec.cin, 32);
                e->steps[ds_step].fused = true;
            }
            t = ov;
        }
        cur = t;
    }
    // a fused downsample reads its input codes subsampled: its slot must be its own
    for (Step& ds : e->steps) {
        if (!ds.fused) continue;
        Value& x = e->vals[ds.in_val];
        const int k = x.code_index(ds.s_in);
        bool shared = false;
        for (const Step& o : e->steps)
            if (&o != &ds && o.in_val == ds.in_val && o.kind != K_MAXPOOL && o.s_in == ds.s_in) shared = true;
        if (shared) {   // undo: run the downsample as its own launch
            ds.fused = false;
            for (Step& c : e->steps)
                if (c.aux_src == (int)(&ds - &e->steps[0])) c.aux_src = -1;
            e->vals[ds.out_val].need_f32 = true;
            continue;
        }
        x.sub2.resize(x.scales.size(), 0);
        x.sub2[k] = 1;
    }
    e->vals[cur].need_f32 = true;
    e->final_val = cur;
    const Value& fv = e->vals[cur];
    if (fv.c != m.fc_in) return e->fail(strf("final map has %d channels but fc_in=%d", fv.c, m.fc_in));
    for (Value& v : e->vals)
        if (v.scales.size() > 2)
            return e->fail("a tensor feeds more than two distinct activation scales (unsupported)");
    return PTQ8_OK;
}

bool make_map(ptq8_engine* e, CUtensorMap* map, CUtensorMapDataType dt, int rank, void* base, const cuuint64_t* dims,
              const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* estr, CUtensorMapSwizzle swz) {
    auto enc = get_encode();
    if (!enc) {
        e->err = "cuTensorMapEncodeTiled entry point not available";
        return false;
    }
    CUresult r = enc(map, dt, rank, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        e->err = strf("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return false;
    }
    return true;
}


// conv_tc_kernel specializations: [K-chunk 32/64/128][mode][code outputs][residual][fp32 out]
void* g_conv_table[3][2][3][2][2];

// the same with the aux GEMM (mode 1, residual): [K-chunk 64/128][code outputs 1/2][fp32 out]
void* g_conv_aux_table[2][2][2];

// Mode 1 with a whole-output N tile of 64 channels, codes only, and the fast epilogue:
// [(K chunk, N tile) = (64, 64), (32, 64) (the stem GEMM)][code outputs 1/2].  (Measured at
// batch 8192: as fast as the general epilogue with a fifth fewer instructions for these
// convs; slower for residual convs, whose column-stationary general epilogue keeps more
// residual loads in flight, and for 128-channel tiles, whose unrolled epilogue is larger.)
void* g_conv_fast_table[2][2];
int fast_index(int cb, int bn) {
    if (cb == 64 && bn == 64) return 0;
    if (cb == 32 && bn == 64) return 1;
    return -1;
}

template <int CBI, int MODE, int NOUT, int RES, int F32>
void fill_one() {
    g_conv_table[CBI][MODE][NOUT][RES][F32] =
        reinterpret_cast<void*>(&conv_tc_kernel<(32 << CBI), MODE, NOUT, RES != 0, F32 != 0, false>);
}
template <int CBI, int NOUT, int F32>
void fill_aux() {
    g_conv_aux_table[CBI - 1][NOUT - 1][F32] =
        reinterpret_cast<void*>(&conv_tc_kernel<(32 << CBI), 1, NOUT, true, F32 != 0, true>);
}
template <int CBI, int MODE, int NOUT, int RES>
void fill_f32() { fill_one<CBI, MODE, NOUT, RES, 0>(); fill_one<CBI, MODE, NOUT, RES, 1>(); }
template <int CB, int FBN, int NOUT>
void fill_fast() {
    g_conv_fast_table[fast_index(CB, FBN)][NOUT - 1] =
        reinterpret_cast<void*>(&conv_tc_kernel<CB, 1, NOUT, false, false, false, FBN>);
}
template <int CBI, int MODE, int NOUT>
void fill_res() { fill_f32<CBI, MODE, NOUT, 0>(); fill_f32<CBI, MODE, NOUT, 1>(); }
template <int CBI, int MODE>
void fill_nout() { fill_res<CBI, MODE, 0>(); fill_res<CBI, MODE, 1>(); fill_res<CBI, MODE, 2>(); }
template <int CBI>
void fill_mode() { fill_nout<CBI, 0>(); fill_nout<CBI, 1>(); }
// The same compile-time N tile epilogue for 64-channel residual convs of the halo-block
// pipeline whose residual is loaded and whose outputs are codes only: [code outputs 1/2].
// (Measured at batch 8192: layer1.1.conv2 0.913 -> 0.889 ms against the column-stationary
// epilogue; with an fp32 output and the aux-GEMM identity, layer1.0.conv2, it was slower,
// 0.78 -> 1.05 ms, and keeps the column-stationary epilogue.)
void* g_conv_fast_res_table[2];
template <int NOUT>
void fill_fast_res() {
    g_conv_fast_res_table[NOUT - 1] = reinterpret_cast<void*>(&conv_tc_kernel<64, 1, NOUT, true, false, false, 64>);
}

// Mode 2 (stride-2 3x3 convs over 64-byte pixels, pixel-pair boxes), codes-only outputs:
// [code outputs 1/2].
void* g_conv_pair_table[2];
template <int NOUT>
void fill_pair() {
    g_conv_pair_table[NOUT - 1] = reinterpret_cast<void*>(&conv_tc_kernel<64, 2, NOUT, false, false, false>);
}

void fill_table() {
    static bool done = false;
    if (done) return;
    fill_pair<1>(); fill_pair<2>();
    fill_fast_res<1>(); fill_fast_res<2>();
    fill_mode<0>();
    fill_mode<1>();
    fill_mode<2>();
    fill_aux<1, 1, 0>(); fill_aux<1, 1, 1>(); fill_aux<1, 2, 0>(); fill_aux<1, 2, 1>();
    fill_aux<2, 1, 0>(); fill_aux<2, 1, 1>(); fill_aux<2, 2, 0>(); fill_aux<2, 2, 1>();
    fill_fast<64, 64, 1>(); fill_fast<64, 64, 2>(); fill_fast<32, 64, 1>(); fill_fast<32, 64, 2>();
    done = true;
}

int cb_index(int cb) { return cb == 128 ? 2 : (cb == 64 ? 1 : 0); }

// Dynamic shared memory of conv_tc_kernel for a pipeline shape (aux_kb > 0: + aux weights [bn][aux_kb]).
size_t conv_smem_bytes(int a_stage, int cb, int bn, int stages, int b_chunks, int aux_kb = 0) {
    const size_t sb = (size_t)round_up(bn * cb, 1024);
    return 1024 + (size_t)stages * a_stage + (size_t)b_chunks * sb + (aux_kb ? (size_t)round_up(bn * aux_kb, 1024) : 0);
}

// Keep the whole weight slab of the N tile resident when it fits next to a
// pipeline of at least `min_res` A stages; otherwise stream weights with A.
// Returns false when mode 1 (which needs resident weights) does not fit.
bool choose_pipeline(Step& st, int min_res) {
    for (int S : {24, 20, 16, 12, 10, 8, 6, 5, 4, 3, 2}) {
        if (S < min_res) break;
        if ((size_t)S * st.a_stage > 96 * 1024 && S > min_res) continue;   // ~96 KB of A in flight is plenty
        const size_t b = conv_smem_bytes(st.a_stage, st.cb, st.bn, S, st.n_kchunks, st.aux_src >= 0 ? st.aux_kb : 0);
        if (b <= kSmemBudget) {
            st.stages = S;
            st.b_resident = 1;
            st.smem = b;
            return true;
        }
    }
    if (st.mode == 1) return false;
    for (int S : {16, 12, 10, 8, 6, 5, 4, 3, 2}) {
        const size_t b = conv_smem_bytes(st.a_stage, st.cb, st.bn, S, S);
        if (b <= kSmemBudget) {
            st.stages = S;
            st.b_resident = 0;
            st.smem = b;
            return true;
        }
    }
    st.stages = 2;
    st.b_resident = 0;
    st.smem = conv_smem_bytes(st.a_stage, st.cb, st.bn, 2, 2);
    return true;
}

int acc_cols_for(int bn) {
    int tc = 32;
    while (tc < bn) tc <<= 1;
    return tc;
}

// Accumulator buffers in TMEM (512 columns) of `cols` columns each: 8 of <= 64
// columns, 4 of 128, 2 of 256.  The epilogue has min(4, buffers) warp groups, each
// owning every n_groups-th buffer -- except for residual convs with N tiles of 49..64
// channels, where all 16 epilogue warps take every tile, each warp a fixed 16-channel
// slice (column-stationary: the slice's dequantization constants stay in registers;
// measured faster only where the per-value work is large enough to pay for every
// warp waiting on every tile).
int n_acc_for(int cols) { return std::min(8, 512 / cols); }
int n_groups_for(int cols, int bn, bool res) {
    if (res && bn > 48 && bn <= 64) return 1;
    // 65..128-channel N tiles: two groups of 8 warps (two slices per lane quadrant), each
    // double-buffering its accumulators, against four groups of 4 warps at batch 8192:
    // layer2.1.conv2 0.668 -> 0.642 ms, layer2.1.conv1 0.286 -> 0.277 ms, layer2.0.conv1
    // 0.248 -> 0.240 ms
    if (bn > 64 && bn <= 128) return std::min(2, n_acc_for(cols));
    return std::min(4, n_acc_for(cols));
}

int finalize(ptq8_engine* e, int max_batch) {
    const Model& m = *e->model;
    if (!e->built) return e->fail("engine not built");
    if (!e->calibrated) return e->fail("calibration ranges not set (set_calib)");
    if (max_batch <= 0) return e->fail("max_batch must be positive");
    if (!e->cuda_ok(cudaSetDevice(e->device), "cudaSetDevice")) return PTQ8_ERR_CUDA;
    if (e->copy_stream) cudaStreamSynchronize(e->copy_stream);
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
    for (void* p : e->allocs) cudaFree(p);
    e->allocs.clear();
    e->d_input2 = nullptr;
    e->d_err = nullptr;
    e->async_slot = 0;
    e->planned = false;
    int rc = plan(e);
    if (rc) return rc;
    if (!e->dalloc(&e->d_err, sizeof(int), "alloc device error word") ||
        !e->cuda_ok(cudaMemset(e->d_err, 0, sizeof(int)), "clear device error word"))
        return PTQ8_ERR_CUDA;
    const size_t NB = (size_t)max_batch;
    // the kernels decode positions in 32-bit arithmetic
    for (const Value& v : e->vals)
        if (NB * (v.h + 2) * (v.w + 2) >= (size_t)1 << 31)
            return e->fail(strf("max_batch %d too large for a %dx%d map (positions must stay below 2^31)", max_batch,
                                v.h, v.w));

    // activation buffers
    for (size_t vi = 0; vi < e->vals.size(); ++vi) {
        Value& v = e->vals[vi];
        const size_t pix = NB * v.h * v.w;
        v.codes.assign(v.scales.size(), nullptr);
        if (vi == 0) continue;   // network input lives in d_input
        // fp32 maps use the f32_off layout: whole 32-position blocks
        if (v.need_f32 && !e->dalloc(&v.f32, ((pix + 31) & ~(size_t)31) * v.c * sizeof(float), "alloc fp32 activation"))
            return PTQ8_ERR_CUDA;
        // int8 codes carry a one-pixel zero border (written once, never touched again);
        // subsampled slots hold the even positions only, in a half-size bordered map
        for (size_t k = 0; k < v.scales.size(); ++k) {
            const size_t bpix = v.is_sub((int)k) ? NB * (v.sub_h() + 2) * (v.sub_w() + 2) : NB * (v.h + 2) * (v.w + 2);
            if (!e->dalloc(&v.codes[k], bpix * v.ldq, "alloc int8 codes")) return PTQ8_ERR_CUDA;
            if (!e->cuda_ok(cudaMemset(v.codes[k], 0, bpix * v.ldq), "clear codes")) return PTQ8_ERR_CUDA;
        }
    }
    if (!e->dalloc(&e->d_input, NB * e->in_c * e->in_h * e->in_w * sizeof(float), "alloc input")) return PTQ8_ERR_CUDA;
    if (!e->dalloc(&e->d_logits, NB * m.fc_out * sizeof(float), "alloc logits")) return PTQ8_ERR_CUDA;
    if (!e->dalloc(&e->d_fc_w, m.fc_w.size() * sizeof(float), "alloc fc") ||
        !e->dalloc(&e->d_fc_b, m.fc_b.size() * sizeof(float), "alloc fc"))
        return PTQ8_ERR_CUDA;
    cudaMemcpy(e->d_fc_w, m.fc_w.data(), m.fc_w.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(e->d_fc_b, m.fc_b.data(), m.fc_b.size() * 4, cudaMemcpyHostToDevice);

    // per-step weights, epilogue constants and tensor maps
    for (Step& st : e->steps) {
        if (st.kind == K_MAXPOOL) continue;
        const ConvQ& cq = e->q[st.conv];
        const ConvSpec& c = cq.spec;
        std::vector<float> factor(c.cout);
        const float s32 = (float)st.s_in;
        for (int o = 0; o < c.cout; ++o) factor[o] = s32 * cq.wscale[o];
        if (!e->dalloc(&st.d_factor, c.cout * 4, "alloc factor") || !e->dalloc(&st.d_bias, c.cout * 4, "alloc bias"))
            return PTQ8_ERR_CUDA;
        cudaMemcpy(st.d_factor, factor.data(), c.cout * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(st.d_bias, cq.bias.data(), c.cout * 4, cudaMemcpyHostToDevice);
        st.h_factor = factor;
        st.h_bias = cq.bias;
        const int K = c.cin * c.kh * c.kw;
        {
            long bound = 0;   // codes are in [-128, 127], so |acc| <= 128 * sum_k |w[c][k]|
            for (int o = 0; o < c.cout; ++o) {
                long sw = 0;
                for (int k = 0; k < K; ++k) sw += std::abs((int)cq.codes[(size_t)o * K + k]);
                bound = std::max(bound, 128 * sw);
            }
            st.acc_small = bound < (1L << 22);
        }
        if (st.kind == K_DW) {
            std::vector<int8_t> w((size_t)c.kh * c.kw * c.cout);
            for (int o = 0; o < c.cout; ++o)
                for (int t = 0; t < c.kh * c.kw; ++t) w[(size_t)t * c.cout + o] = cq.codes[(size_t)o * K + t];
            if (!e->dalloc(&st.d_w, w.size(), "alloc dw weights")) return PTQ8_ERR_CUDA;
            cudaMemcpy(st.d_w, w.data(), w.size(), cudaMemcpyHostToDevice);
            if (dw3x3_eligible(e, st)) {
                // word (j, c) of group g: column j of channel 4g + c, bytes (w[0][j], w[1][j], w[2][j], 0)
                const int G4 = (c.cout + 3) / 4;
                std::vector<uint32_t> t((size_t)G4 * 12, 0u);
                auto code = [&](int o, int tap) { return (uint32_t)(uint8_t)cq.codes[(size_t)o * K + tap]; };
                for (int o = 0; o < c.cout; ++o)
                    for (int j = 0; j < 3; ++j)
                        t[(size_t)(o / 4) * 12 + 4 * j + o % 4] = code(o, j) | code(o, 3 + j) << 8 | code(o, 6 + j) << 16;
                if (cq.bits == 4) {
                    // W4: each word as 16 bits, its three codes in nibbles 0-2 (24 bytes per group)
                    std::vector<uint16_t> h(t.size());
                    for (size_t k = 0; k < t.size(); ++k)
                        h[k] = (uint16_t)((t[k] & 0xF) | ((t[k] >> 4) & 0xF0) | ((t[k] >> 8) & 0xF00));
                    if (!e->dalloc(&st.d_dwt, h.size() * 2, "alloc dw table")) return PTQ8_ERR_CUDA;
                    cudaMemcpy(st.d_dwt, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
                    st.w_packed = true;
                    st.w_dev_bytes = h.size() * 2;
                } else {
                    if (!e->dalloc(&st.d_dwt, t.size() * 4, "alloc dw table")) return PTQ8_ERR_CUDA;
                    cudaMemcpy(st.d_dwt, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
                    st.w_dev_bytes = t.size() * 4;
                }
            } else {
                st.w_dev_bytes = w.size();
            }
            continue;
        }
        // tensor-core conv: weight matrix [cout][ktot] int8, K-major
        std::vector<int8_t> w;
        int cpad;
        if (st.kind == K_STEM_IM2COL) {
            st.kpad = round_up(K, 32);
            cpad = st.kpad;
            st.ktot = st.kpad;
            w.assign((size_t)c.cout * st.ktot, 0);
            for (int o = 0; o < c.cout; ++o)
                for (int ci = 0; ci < c.cin; ++ci)
                    for (int i = 0; i < c.kh; ++i)
                        for (int j = 0; j < c.kw; ++j)
                            w[(size_t)o * st.ktot + (i * c.kw + j) * c.cin + ci] =
                                cq.codes[(((size_t)o * c.cin + ci) * c.kh + i) * c.kw + j];
            const size_t rows = NB * (st.oh + 2) * (st.ow + 2);
            if (!e->dalloc(&st.d_im2col, rows * st.kpad, "alloc im2col") ||
                !e->cuda_ok(cudaMemset(st.d_im2col, 0, rows * st.kpad), "clear im2col"))
                return PTQ8_ERR_CUDA;
        } else {
            cpad = round_up(c.cin, 32);
            st.ktot = c.kh * c.kw * cpad;
            w.assign((size_t)c.cout * st.ktot, 0);
            for (int o = 0; o < c.cout; ++o)
                for (int ci = 0; ci < c.cin; ++ci)
                    for (int i = 0; i < c.kh; ++i)
                        for (int j = 0; j < c.kw; ++j)
                            w[(size_t)o * st.ktot + (i * c.kw + j) * cpad + ci] =
                                cq.codes[(((size_t)o * c.cin + ci) * c.kh + i) * c.kw + j];
        }
        st.cb = choose_cb(cpad);
        choose_bn(c.cout, &st.bn, &st.n_ntiles);
        if (round_up(c.cout, 32) > kMaxConstCh)
            return e->fail(strf("conv[%d]: %d output channels exceed the kernel's %d", st.conv, c.cout, kMaxConstCh));
        if (st.n_ntiles > 1 && st.bn % 32 != 0)
            return e->fail(strf("conv[%d]: N tile %d breaks the 32-byte store alignment", st.conv, st.bn));
        if (st.fused) {   // weights and constants are read (as int8, by TMA) by the conv that computes it
            if (!e->dalloc(&st.d_w, w.size(), "alloc weights")) return PTQ8_ERR_CUDA;
            cudaMemcpy(st.d_w, w.data(), w.size(), cudaMemcpyHostToDevice);
            st.w_dev_bytes = w.size();
            continue;
        }
        tile_shape(max_batch, st.oh, st.ow, &st.TW, &st.TH, &st.TN);
        if (cq.pos_tiles) {   // one output position of 128 images per M tile
            st.TW = st.TH = 1;
            st.TN = 128;
        }
        st.n_kchunks = st.kind == K_STEM_IM2COL ? st.kpad / st.cb : st.kh * st.kw * (cpad / st.cb);
        // mode 1: stride-1 "same" convs read one halo block per tile (needs resident weights)
        st.mode = 0;
        // (the kernel's halo-block MMA loop is compiled for 3x3)
        if (st.kind == K_TC && cq.view_oh == 0 && !cq.pos_tiles && st.kh == 3 && st.kw == 3 && st.sh == 1 && st.sw == 1 &&
            st.ph == (st.kh - 1) / 2 && st.pw == st.ph && st.ph <= 1 && st.oh == st.ih && st.ow == st.iw &&
            st.oh * st.ow >= 64) {
            const int wp = st.iw + 2;
            st.blk_rows = 128 + (st.kh - 1) * wp + (st.kw - 1);
            if (st.blk_rows <= 256) {
                st.mode = 1;
                st.a_stage = round_up(st.blk_rows * st.cb, 1024);
                if (st.aux_src >= 0) {   // + the aux tile: 128 rows of aux_kb bytes
                    st.aux_off = st.a_stage;
                    st.a_stage += 128 * st.aux_kb;
                }
                if (!choose_pipeline(st, 2)) st.mode = 0;
            }
        }
        // mode 2: a stride-2 3x3 conv over 64-byte pixels (64 channels) reads, per kernel row, one
        // 4-D box of pixel pairs (2w, 2w+1) -- taps 0 and 1 in its two 64-byte halves -- and one of
        // the pairs one further (tap 2 in the first half): 6 boxes of 128 rows x 128 bytes per tile
        // instead of 9 of 64-byte rows, whose per-row cost bounds these convs.  Needs resident
        // weights and a codes-only output.
        if (st.kind == K_TC && st.mode == 0 && cq.view_oh == 0 && !cq.pos_tiles && st.kh == 3 && st.kw == 3 &&
            st.sh == 2 && st.sw == 2 && st.ph == 1 && st.pw == 1 && cpad == 64 && st.cb == 64 &&
            e->vals[st.in_val].ldq == 64 && (st.iw + 2) % 2 == 0 && st.aux_src < 0 && st.res_val < 0 &&
            !e->vals[st.out_val].need_f32 && e->vals[st.out_val].scales.size() >= 1 &&
            e->vals[st.out_val].scales.size() <= 2 && st.TW * st.TH * st.TN == 128) {
            st.mode = 2;
            st.a_stage = 128 * 128;
            if (!choose_pipeline(st, 2) || !st.b_resident) st.mode = 0;
        }
        if (st.kind == K_STEM_IM2COL) {
            // the stem GEMM reads its bordered im2col rows as a 1x1 conv: tiles of 128 consecutive
            // bordered rows, one 2-D box each (4-D boxes of 32-byte rows were several times slower)
            st.blk_rows = 128;
            st.mode = 1;
            st.a_stage = round_up(st.blk_rows * st.cb, 1024);
            if (!choose_pipeline(st, 2)) st.mode = 0;
        }
        if (st.aux_src >= 0 && (st.mode != 1 || st.n_ntiles != 1 || (st.cb != 64 && st.cb != 128)))
            return e->fail(strf("conv[%d]: residual fusion needs the halo-block pipeline", st.conv));
        st.acc_cols = acc_cols_for(st.bn) * (st.aux_src >= 0 ? 2 : 1);
        if (st.mode == 0) {
            st.a_stage = 128 * st.cb;
            choose_pipeline(st, 4);
        }
        if (st.smem > kSmemBudget)
            return e->fail(strf("conv[%d]: no pipeline fits in shared memory", st.conv));
        // Weights in HBM: W4 codes of a resident slab two per byte (unpacked into shared memory
        // by the kernel); otherwise the int8 matrix, loaded by TMA.  The stem's weights stay
        // int8: layer1.0.conv2's aux GEMM reads them with TMA.
        st.w_packed = cq.bits == 4 && st.kind == K_TC && st.b_resident;
        if (st.w_packed) {
            std::vector<uint8_t> p(w.size() / 2);
            for (size_t k = 0; k < p.size(); ++k)
                p[k] = (uint8_t)((w[2 * k] & 0x0F) | ((w[2 * k + 1] & 0x0F) << 4));
            if (!e->dalloc(&st.d_w4, p.size(), "alloc packed weights")) return PTQ8_ERR_CUDA;
            cudaMemcpy(st.d_w4, p.data(), p.size(), cudaMemcpyHostToDevice);
            st.w_dev_bytes = p.size();
        } else {
            if (!e->dalloc(&st.d_w, w.size(), "alloc weights")) return PTQ8_ERR_CUDA;
            cudaMemcpy(st.d_w, w.data(), w.size(), cudaMemcpyHostToDevice);
            st.w_dev_bytes = w.size();
            cuuint64_t dims[2] = {(cuuint64_t)st.ktot, (cuuint64_t)c.cout};
            cuuint64_t strides[1] = {(cuuint64_t)st.ktot};
            cuuint32_t box[2] = {(cuuint32_t)st.cb, (cuuint32_t)st.bn};
            cuuint32_t estr[2] = {1, 1};
            if (!make_map(e, &st.map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, st.d_w, dims, strides, box, estr,
                          swizzle_for(st.cb)))
                return PTQ8_ERR_CUDA;
        }
        if (st.kind == K_STEM_IM2COL && st.mode == 1) {
            const cuuint64_t rows = (cuuint64_t)max_batch * (st.oh + 2) * (st.ow + 2);
            cuuint64_t dims[2] = {(cuuint64_t)st.kpad, rows};
            cuuint64_t strides[1] = {(cuuint64_t)st.kpad};
            cuuint32_t box[2] = {(cuuint32_t)st.cb, (cuuint32_t)st.blk_rows};
            cuuint32_t estr[2] = {1, 1};
            if (!make_map(e, &st.map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, st.d_im2col, dims, strides, box, estr,
                          swizzle_for(st.cb)))
                return PTQ8_ERR_CUDA;
        } else if (st.kind == K_STEM_IM2COL) {
            // the im2col rows form a bordered [N][OH+2][OW+2][kpad] map read as a 1x1 conv
            const cuuint64_t hp = st.oh + 2, wp = st.ow + 2;
            cuuint64_t dims[4] = {(cuuint64_t)st.kpad, wp, hp, (cuuint64_t)max_batch};
            cuuint64_t strides[3] = {(cuuint64_t)st.kpad, (cuuint64_t)st.kpad * wp, (cuuint64_t)st.kpad * wp * hp};
            cuuint32_t box[4] = {(cuuint32_t)st.cb, (cuuint32_t)st.TW, (cuuint32_t)st.TH, (cuuint32_t)st.TN};
            cuuint32_t estr[4] = {1, 1, 1, 1};
            if (!make_map(e, &st.map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, st.d_im2col, dims, strides, box, estr,
                          swizzle_for(st.cb)))
                return PTQ8_ERR_CUDA;
        } else if (st.mode == 1) {
            const Value& vin = e->vals[st.in_val];
            int8_t* base = vin.codes[vin.code_index(st.s_in)];
            const cuuint64_t rows = (cuuint64_t)max_batch * (vin.h + 2) * (vin.w + 2);
            cuuint64_t dims[2] = {(cuuint64_t)vin.c, rows};
            cuuint64_t strides[1] = {(cuuint64_t)vin.ldq};
            cuuint32_t box[2] = {(cuuint32_t)st.cb, (cuuint32_t)st.blk_rows};
            cuuint32_t estr[2] = {1, 1};
            if (!make_map(e, &st.map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr,
                          swizzle_for(st.cb)))
                return PTQ8_ERR_CUDA;
            if (st.aux_src >= 0) {
                // aux rows aligned with this conv's bordered tile rows: the stem's bordered
                // im2col rows, or the subsampled block-input codes of a fused downsample
                const Step& src = e->steps[st.aux_src];
                const int kb = st.aux_kb;
                void* xbase = nullptr;
                cuuint64_t xc = 0, xld = 0;
                if (src.kind == K_STEM_IM2COL) {
                    if (src.oh != vin.h || src.ow != vin.w || src.kpad != 32 || kb != 32 || !src.d_im2col)
                        return e->fail(strf("conv[%d]: stem identity fusion geometry mismatch", st.conv));
                    xbase = src.d_im2col;
                    xc = 32;
                    xld = 32;
                } else {
                    const Value& x = e->vals[src.in_val];
                    const int k = x.code_index(src.s_in);
                    if (!x.is_sub(k) || x.sub_h() != vin.h || x.sub_w() != vin.w || round_up(x.c, 32) != kb)
                        return e->fail(strf("conv[%d]: downsample fusion geometry mismatch", st.conv));
                    xbase = x.codes[k];
                    xc = (cuuint64_t)x.c;
                    xld = (cuuint64_t)x.ldq;
                }
                if (!src.d_w) return e->fail(strf("conv[%d]: aux weights missing", st.conv));
                cuuint64_t xdims[2] = {xc, rows};
                cuuint64_t xstr[1] = {xld};
                cuuint32_t xbox[2] = {(cuuint32_t)kb, 128};
                if (!make_map(e, &st.map_xa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xbase, xdims, xstr, xbox, estr,
                              swizzle_for(kb)))
                    return PTQ8_ERR_CUDA;
                cuuint64_t wdims[2] = {(cuuint64_t)src.ktot, (cuuint64_t)e->q[src.conv].spec.cout};
                cuuint64_t wstr[1] = {(cuuint64_t)src.ktot};
                cuuint32_t wbox[2] = {(cuuint32_t)kb, (cuuint32_t)st.bn};
                if (!make_map(e, &st.map_xb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, src.d_w, wdims, wstr, wbox, estr,
                              swizzle_for(kb)))
                    return PTQ8_ERR_CUDA;
            }
        } else {
            const Value& vin = e->vals[st.in_val];
            int8_t* base = vin.codes[vin.code_index(st.s_in)];
            const cuuint64_t hp = vin.h + 2, wp = vin.w + 2;
            if (st.mode == 2) {   // elements are pixel pairs: 128 bytes of two 64-byte code rows
                cuuint64_t pdims[4] = {128, wp / 2, hp, (cuuint64_t)max_batch};
                cuuint64_t pstrides[3] = {128, (cuuint64_t)vin.ldq * wp, (cuuint64_t)vin.ldq * wp * hp};
                cuuint32_t pbox[4] = {128, (cuuint32_t)st.TW, (cuuint32_t)(st.TH * 2), (cuuint32_t)st.TN};
                cuuint32_t pestr[4] = {1, 1, 2, 1};
                if (pbox[2] > 256 || !make_map(e, &st.map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, pdims, pstrides,
                                                pbox, pestr, swizzle_for(128)))
                    return pbox[2] > 256 ? e->fail(strf("conv[%d]: pair box taller than 256 rows", st.conv))
                                         : PTQ8_ERR_CUDA;
                continue;
            }
            cuuint64_t dims[4] = {(cuuint64_t)vin.c, wp, hp, (cuuint64_t)max_batch};
            cuuint64_t strides[3] = {(cuuint64_t)vin.ldq, (cuuint64_t)vin.ldq * wp, (cuuint64_t)vin.ldq * wp * hp};
            cuuint32_t box[4] = {(cuuint32_t)st.cb, (cuuint32_t)(st.TW * st.sw), (cuuint32_t)(st.TH * st.sh),
                                 (cuuint32_t)st.TN};
            cuuint32_t estr[4] = {1, (cuuint32_t)st.sw, (cuuint32_t)st.sh, 1};
            if (box[1] > 256 || box[2] > 256 || st.sw > 8 || st.sh > 8)
                return e->fail(strf("conv[%d]: tile/stride outside the TMA box limits", st.conv));
            if (!make_map(e, &st.map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, dims, strides, box, estr,
                          swizzle_for(st.cb)))
                return PTQ8_ERR_CUDA;
        }
    }
    {
        fill_table();
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, e->device);
        for (Step& st : e->steps) {
            if ((st.kind != K_TC && st.kind != K_STEM_IM2COL) || st.fused) continue;
            const Value& out = e->vals[st.out_val];
            const int nout = (int)out.scales.size();
            const int res = st.res_val >= 0 ? 1 : 0;
            const int f32 = out.need_f32 ? 1 : 0;
            // the compile-time N tile epilogue: halo-block mode, one N tile holding all 64 output
            // channels, codes only (no residual, fp32 map or aux GEMM)
            st.fast = (st.kind == K_TC || st.kind == K_STEM_IM2COL) && st.mode == 1 && st.n_ntiles == 1 &&
                      e->q[st.conv].view_oh == 0 && st.oc == st.bn && fast_index(st.cb, st.bn) >= 0 &&
                      nout >= 1 && nout <= 2 && !res && !f32 && st.aux_src < 0;
            const bool fast_res = !st.fast && st.kind == K_TC && st.mode == 1 && st.n_ntiles == 1 &&
                                  e->q[st.conv].view_oh == 0 && st.oc == 64 && st.bn == 64 && st.cb == 64 &&
                                  nout >= 1 && nout <= 2 && res && !f32 && st.aux_src < 0;
            if (fast_res) {
                st.fast = true;
                st.kfn = g_conv_fast_res_table[nout - 1];
            } else if (st.fast) {
                st.kfn = g_conv_fast_table[fast_index(st.cb, st.bn)][nout - 1];
            } else if (st.mode == 2) {
                st.kfn = g_conv_pair_table[nout - 1];
            } else if (st.aux_src >= 0) {
                if (nout < 1 || nout > 2) return e->fail(strf("conv[%d]: stem identity fusion needs 1-2 code outputs", st.conv));
                st.kfn = g_conv_aux_table[cb_index(st.cb) - 1][nout - 1][f32];
            } else {
                st.kfn = g_conv_table[cb_index(st.cb)][st.mode][nout][res][f32];
            }
            if (!e->cuda_ok(cudaFuncSetAttribute(st.kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget),
                            "smem attr"))
                return PTQ8_ERR_CUDA;
            int occ = 1;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, st.kfn, kConvThreads, st.smem);
            const int occ_tmem = 512 / (n_acc_for(st.acc_cols) * st.acc_cols);
            occ = std::max(1, std::min(occ, occ_tmem));
            st.grid_x = std::max(1, sms * occ / st.n_ntiles);
        }
        // A kernel's shared-memory limit is a property of the function, shared by every
        // engine of the process: always the same value, covering every plan.
        for (Step& st : e->steps) {
            if (st.kind != K_DW || !st.d_dwt) continue;
            if (!plan_dw3x3(e, st, max_batch)) {
                st.d_dwt = nullptr;   // no tiling fits: the generic depthwise kernel runs it
                st.w_packed = false;  // (with its int8 weights)
                st.w_dev_bytes = (size_t)st.kh * st.kw * st.oc;
                continue;
            }
            if (!e->cuda_ok(cudaFuncSetAttribute(st.dw_kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kDwSmemLimit),
                            "dw smem attr"))
                return PTQ8_ERR_CUDA;
            int occ = 1;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, st.dw_kfn, st.dw_cons + 32,
                                                          (size_t)st.dw_stages * st.dw_stage);
            st.dw_ctas = std::max(1, occ) * sms;
        }
    }
    if (!e->stream) {
        if (!e->cuda_ok(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream")) return PTQ8_ERR_CUDA;
        e->own_stream = true;
    }
    e->max_batch = max_batch;
    e->planned = true;
    return PTQ8_OK;
}

EpiParams epi_for(ptq8_engine* e, const Step& st) {
    EpiParams p{};
    const Value& out = e->vals[st.out_val];
    p.factor = st.d_factor;
    p.bias = st.d_bias;
    p.residual = st.res_val >= 0 ? e->vals[st.res_val].f32 : nullptr;
    p.out_f32 = out.need_f32 ? out.f32 : nullptr;
    p.cout = st.kind == K_MAXPOOL ? out.c : st.oc;
    p.vec32 = (p.cout % 8 == 0) ? 1 : 0;   // 32-byte aligned fp32 rows
    if (st.conv >= 0 && e->q[st.conv].view_oh > 0) {
        p.dcr_oc = out.c;
        p.dcr_h = out.h;
        p.dcr_w = out.w;
    }
    p.act = st.act;
    p.post = st.res_val >= 0 ? st.post : 0;
    p.acc_small = st.acc_small ? 1 : 0;
    p.out_q0 = out.codes.size() > 0 ? out.codes[0] : nullptr;
    p.out_q1 = out.codes.size() > 1 ? out.codes[1] : nullptr;
    p.ldq0 = p.ldq1 = out.ldq;
    for (int k = 0; k < 2; ++k)
        if (out.is_sub(k)) p.sub_mask |= 1 << k;
    p.sub_h = out.sub_h();
    p.sub_w = out.sub_w();
    if (out.scales.size() > 0) {
        p.s0 = out.scales[0];
        p.inv0 = (float)(1.0 / out.scales[0]);
        p.q0 = make_qparams(out.scales[0]);
    }
    if (out.scales.size() > 1) {
        p.s1 = out.scales[1];
        p.inv1 = (float)(1.0 / out.scales[1]);
        p.q1 = make_qparams(out.scales[1]);
    }
    return p;
}

// Every kernel of the forward is launched with programmatic stream serialization:
// it may be scheduled as soon as the previous kernel's blocks have passed their
// set-up (griddepcontrol.launch_dependents), does its own set-up (barriers, TMEM,
// resident weights, constants) meanwhile, and waits (griddepcontrol.wait) before
// reading anything an earlier kernel wrote.
template <typename... Params, typename... Args>
void launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

// Launch step `si` (si == steps.size(): the pooling head) for batch n on the engine stream.
void enqueue_step(ptq8_engine* e, int n, size_t si) {
    cudaStream_t s = e->stream;
    if (si == e->steps.size()) {
        const Value& fv = e->vals[e->final_val];
        const Model& m = *e->model;
        launch_pdl(head_kernel, dim3(n), dim3(256), fv.c * sizeof(float), s, fv.f32, fv.h * fv.w, fv.c, e->d_fc_w,
                   e->d_fc_b, m.fc_out, e->d_logits);
        return;
    }
    const Step& st = e->steps[si];
    if (st.fused) return;   // computed inside its block's last conv
    EpiParams ep = epi_for(e, st);
    if (st.kind == K_MAXPOOL) {
        const size_t total = (size_t)n * st.oh * st.ow * st.oc;
        const int grid = (int)std::min<size_t>((total + 255) / 256, 148 * 32);
        launch_pdl(maxpool_kernel, dim3(grid), dim3(256), 0, s, e->vals[st.in_val].f32, n, st.ih, st.iw, st.ic, st.oh,
                   st.ow, ep);
        return;
    }
    if (st.kind == K_DW && st.d_dwt) {
        const Value& vin = e->vals[st.in_val];
        DwGeom d{};
        d.G4 = (st.oc + 3) / 4;
        d.C = st.oc;
        d.H = st.ih;
        d.W = st.iw;
        d.OH = st.oh;
        d.OW = st.ow;
        d.ldi = vin.ldq;
        d.N = n;
        d.R = st.dw_R;
        d.k_img = st.dw_kimg;
        d.rows_img = st.dw_rows;
        d.bands = st.oh / st.dw_R;
        d.n_units = st.dw_kimg > 1 ? (n + st.dw_kimg - 1) / st.dw_kimg : n * d.bands;
        d.stage_bytes = st.dw_stage;
        d.n_stages = st.dw_stages;
        d.strips = st.ow / st.dw_T;
        d.fd_strips = make_fastdiv(d.strips);
        d.fd_rs = make_fastdiv(st.dw_R * d.strips);
        d.fd_bands = make_fastdiv(d.bands);
        d.err = e->d_err;
        d.wait_limit = e->wait_limit;
        d.w_packed = st.w_packed ? 1 : 0;
        const int grid = std::max(1, std::min(d.n_units, st.dw_ctas));
        launch_pdl((DwKernel)st.dw_kfn, dim3(grid), dim3(st.dw_cons + 32), (size_t)d.n_stages * d.stage_bytes, s,
                   vin.codes[vin.code_index(st.s_in)], (const uint4*)st.d_dwt, d, ep);
        return;
    }
    if (st.kind == K_DW) {
        const Value& vin = e->vals[st.in_val];
        const int8_t* in = vin.codes[vin.code_index(st.s_in)];
        const size_t total = (size_t)n * st.oh * st.ow * ((st.oc + 3) / 4);
        const int grid = (int)std::min<size_t>((total + 255) / 256, 148 * 64);
        launch_pdl(dw_conv_kernel, dim3(grid), dim3(256), 0, s, in, vin.ldq, st.d_w, n, st.ih, st.iw, st.oc, st.oh, st.ow,
                   st.kh, st.kw, st.sh, st.sw, st.ph, st.pw, ep);
        return;
    }
    if (st.kind == K_STEM_IM2COL && e->q[st.conv].spec.cin == 3 && e->q[st.conv].spec.kh == 3 &&
        e->q[st.conv].spec.kw == 3 && e->q[st.conv].spec.sh == 1 && e->q[st.conv].spec.sw == 1 &&
        e->q[st.conv].spec.ph == 1 && e->q[st.conv].spec.pw == 1 && st.kpad == 32 && st.oh == st.ih &&
        st.ow == st.iw) {
        // the CIFAR stem: pixel-major band, whole images per CTA while the band stays within 24 KB
        int rows = st.oh;
        while (rows > 1 && (size_t)3 * (rows + 2) * (st.iw + 2) > 24 * 1024) rows = (rows + 1) / 2;
        const int bands = (st.oh + rows - 1) / rows;
        const size_t band_bytes = (size_t)3 * (rows + 2) * (st.iw + 2);
        const size_t smem = ((band_bytes + 16 + 15) & ~(size_t)15) + (e->cur_input_u8 ? 3 * 256 : 0);
        const FastDiv fbw = make_fastdiv((uint32_t)(st.iw + 2)), fbh = make_fastdiv((uint32_t)(rows + 2));
        if (e->cur_input_u8)
            launch_pdl(stem_im2col3_kernel<true>, dim3(n * bands), dim3(256), smem, s, (const void*)e->cur_input_u8,
                       st.d_im2col, n, st.ih, st.iw, rows, fbw, fbh, (float)(1.0 / st.s_in), st.s_in, e->u8_norm);
        else
            launch_pdl(stem_im2col3_kernel<false>, dim3(n * bands), dim3(256), smem, s,
                       (const void*)(e->cur_input ? e->cur_input : (const float*)e->d_input), st.d_im2col, n, st.ih,
                       st.iw, rows, fbw, fbh, (float)(1.0 / st.s_in), st.s_in, e->u8_norm);
    } else if (st.kind == K_STEM_IM2COL) {
        const ConvSpec& c = e->q[st.conv].spec;
        // whole images per CTA while the quantized band stays within 24 KB of shared memory
        const size_t band_w = (size_t)(st.ow - 1) * c.sw + c.kw;
        int rows = st.oh;
        while (rows > 1 && (size_t)c.cin * ((rows - 1) * c.sh + c.kh) * band_w > 24 * 1024) rows = (rows + 1) / 2;
        const int bands = (st.oh + rows - 1) / rows;
        const size_t band_bytes =
            (((size_t)c.cin * ((rows - 1) * c.sh + c.kh) * band_w + 15) & ~(size_t)15) + (size_t)st.kpad * sizeof(int);
        if (e->cur_input_u8)   // 8-bit pixels, normalised and quantized through a per-CTA code table
            launch_pdl(stem_im2col_kernel<true>, dim3(n * bands), dim3(256), band_bytes + (size_t)c.cin * 256, s,
                       (const void*)e->cur_input_u8, st.d_im2col, n, c.cin, st.ih, st.iw, st.oh, st.ow, c.kh, c.kw,
                       c.sh, c.sw, c.ph, c.pw, st.kpad, rows, (float)(1.0 / st.s_in), st.s_in, e->u8_norm);
        else
            launch_pdl(stem_im2col_kernel<false>, dim3(n * bands), dim3(256), band_bytes, s,
                       (const void*)(e->cur_input ? e->cur_input : (const float*)e->d_input), st.d_im2col, n, c.cin,
                       st.ih, st.iw, st.oh, st.ow, c.kh, c.kw, c.sh, c.sw, c.ph, c.pw, st.kpad, rows,
                       (float)(1.0 / st.s_in), st.s_in, e->u8_norm);
    }
    ConvGeom g{};
    g.mode = st.mode;
    g.N = n;
    g.OH = st.oh;
    g.OW = st.ow;
    g.TW = st.TW; g.TH = st.TH; g.TN = st.TN;
    g.tiles_w = (st.ow + st.TW - 1) / st.TW;
    g.tiles_h = (st.oh + st.TH - 1) / st.TH;
    g.KH = st.kind == K_STEM_IM2COL ? 1 : st.kh;
    if (st.kind == K_STEM_IM2COL) {
        g.KW = 1; g.KH = 1; g.SH = 1; g.SW = 1; g.PH = 0; g.PW = 0;
        g.coord_off = 1;   // bordered im2col map
        g.n_cchunks = st.kpad / st.cb;
    } else {
        g.KW = st.kw; g.SH = st.sh; g.SW = st.sw; g.PH = st.ph; g.PW = st.pw;
        g.coord_off = 1;
        g.n_cchunks = e->vals[st.in_val].ldq / st.cb;
        g.pos_tiles = st.mode == 0 && e->q[st.conv].pos_tiles ? 1 : 0;
        g.IH = st.ih;
        g.IW = st.iw;
    }
    if (st.mode == 1) {
        // the bordered grid of the output (= of the input for stride-1 "same" convs; the stem's
        // im2col rows share its output's grid)
        g.Hp = st.oh + 2;
        g.Wp = st.ow + 2;
        g.blk_off = st.kind == K_STEM_IM2COL ? 0 : -(st.ph * g.Wp + st.pw);
        g.m_tiles = (int)(((size_t)n * g.Hp * g.Wp + 127) / 128);
        g.a_bytes = (uint32_t)(st.blk_rows * st.cb);
    } else {
        g.m_tiles = g.tiles_w * g.tiles_h * ((n + st.TN - 1) / st.TN);
        g.a_bytes = (uint32_t)(st.TW * st.TH * st.TN * (st.mode == 2 ? 128 : st.cb));
    }
    g.a_stage = st.a_stage;
    g.n_kchunks = st.n_kchunks;
    g.fd_img = make_fastdiv((uint32_t)(g.Hp * g.Wp));
    g.fd_wp = make_fastdiv((uint32_t)g.Wp);
    g.fd_tiles_w = make_fastdiv((uint32_t)g.tiles_w);
    g.fd_tiles_h = make_fastdiv((uint32_t)g.tiles_h);
    g.BN = st.bn;
    g.acc_cols = st.acc_cols;
    g.n_acc = n_acc_for(st.acc_cols);
    g.n_groups = st.fast ? std::min(4, g.n_acc) : n_groups_for(st.acc_cols, st.bn, st.res_val >= 0);
    if (st.aux_src >= 0) {
        const Step& src = e->steps[st.aux_src];
        g.aux_off = st.aux_off;
        g.aux_bytes = (uint32_t)(128 * st.aux_kb);
        g.aux_kb = st.aux_kb;
        g.aux_col = acc_cols_for(st.bn);
        ep.aux_act = src.act;
    }
    g.stages = st.stages;
    g.b_resident = st.b_resident;
    g.b_bytes = (uint32_t)(st.bn * st.cb);
    g.err = e->d_err;
    g.wait_limit = e->wait_limit;
    g.w4 = st.d_w4;
    g.w4_ld = st.ktot / 2;
    g.w_rows = e->q[st.conv].spec.cout;
    g.b_packed = st.w_packed ? 1 : 0;
    g.stall_first_load = 0;
    if (e->stall_first_load) {   // the forward's first tensor-core conv only
        size_t first = e->steps.size();
        for (size_t k = 0; k < e->steps.size() && first == e->steps.size(); ++k)
            if ((e->steps[k].kind == K_TC || e->steps[k].kind == K_STEM_IM2COL) && !e->steps[k].fused) first = k;
        g.stall_first_load = si == first ? 1 : 0;
    }
    const int gx = e->max_ctas > 0 ? std::min(st.grid_x, std::max(1, e->max_ctas / st.n_ntiles)) : st.grid_x;
    dim3 grid((unsigned)std::min(g.m_tiles, gx), (unsigned)st.n_ntiles);
    CUtensorMap ma = st.map_a, mb = st.map_b, mxa = st.map_xa, mxb = st.map_xb;
    std::unique_ptr<ConvConsts> cc(new ConvConsts());   // zero past cout
    for (size_t c = 0; c < st.h_factor.size(); ++c) cc->fb[c] = make_float2(st.h_factor[c], st.h_bias[c]);
    if (st.aux_src >= 0) {
        const Step& src = e->steps[st.aux_src];
        for (size_t c = 0; c < src.h_factor.size(); ++c) cc->aux_fb[c] = make_float2(src.h_factor[c], src.h_bias[c]);
    }
    void* args[7] = {&ma, &mb, &mxa, &mxb, &g, &ep, cc.get()};
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kConvThreads);
    cfg.dynamicSmemBytes = st.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelExC(&cfg, st.kfn, args);
}

int enqueue(ptq8_engine* e, int n) {
    for (size_t si = 0; si <= e->steps.size(); ++si) enqueue_step(e, n, si);
    if (!e->cuda_ok(cudaGetLastError(), "kernel launch")) return PTQ8_ERR_CUDA;
    return PTQ8_OK;
}

// Algorithmic work of step si for batch n: multiply-accumulates and the bytes a
// perfect kernel moves (input codes once, weights once, every output once).
void step_work(const ptq8_engine* e, int n, size_t si, double* macs, double* bytes, int* kind) {
    if (si == e->steps.size()) {
        const Value& fv = e->vals[e->final_val];
        *kind = 4;
        *macs = (double)n * e->model->fc_in * e->model->fc_out;
        *bytes = (double)n * fv.h * fv.w * fv.c * 4.0 + (double)n * e->model->fc_out * 4.0;
        return;
    }
    const Step& st = e->steps[si];
    *kind = st.kind;
    if (st.fused) {   // counted with the conv that computes it
        *macs = 0;
        *bytes = 0;
        return;
    }
    const Value& out = e->vals[st.out_val];
    double outb = 0;
    for (size_t k = 0; k < out.scales.size(); ++k)
        outb += (double)n * (out.is_sub((int)k) ? out.sub_h() * out.sub_w() : out.h * out.w) * out.c;
    if (out.need_f32) outb += (double)n * out.h * out.w * out.c * 4.0;
    // residual: the stored fp32 map, or (aux GEMM) the aux rows (stem im2col / subsampled codes)
    double resb = st.res_val < 0 ? 0.0
                  : st.aux_src >= 0 ? (double)n * (out.h + 2) * (out.w + 2) * st.aux_kb
                                    : (double)n * out.h * out.w * out.c * 4.0;
    if (st.kind == K_MAXPOOL) {
        *macs = 0;
        *bytes = (double)n * st.ih * st.iw * st.ic * 4.0 + outb;
        return;
    }
    const ConvSpec& c = e->q[st.conv].spec;
    const double pos = (double)n * st.oh * st.ow;
    *macs = pos * c.cout * (double)c.cin * c.kh * c.kw;
    const double inb = st.kind == K_STEM_IM2COL ? (double)n * st.ih * st.iw * st.ic * 4.0
                                                : (double)n * st.ih * st.iw * st.ic;
    // weights once: W4 codes held two per byte count half a byte each
    *bytes = inb + (st.w_packed ? 0.5 : 1.0) * c.cout * c.cin * c.kh * c.kw + outb + resb;
    if (st.aux_src >= 0 && e->steps[st.aux_src].fused) {   // the downsample's GEMM runs here
        const ConvSpec& d = e->q[e->steps[st.aux_src].conv].spec;
        *macs += pos * d.cout * (double)d.cin;
        *bytes += (double)d.cout * d.cin;
    }
}

// The CUDA graph of one forward at batch n reading input slot `slot` (0: d_input,
// 1: d_input2; u8: the 8-bit pixel slots d_input_u8[slot]), captured on first use,
// then cached.
int graph_for(ptq8_engine* e, int n, cudaGraphExec_t* out, int slot = 0, bool u8 = false) {
    if (!e->planned) {
        int rc = finalize(e, std::max(n, e->max_batch > 0 ? e->max_batch : n));
        if (rc) return rc;
    }
    if (n <= 0 || n > e->max_batch)
        return e->fail(strf("batch %d outside [1, %d] (alloc_scratch sets the maximum)", n, e->max_batch));
    if (!e->cuda_ok(cudaSetDevice(e->device), "cudaSetDevice")) return PTQ8_ERR_CUDA;
    if (u8 && !e->d_input_u8[slot]) return e->fail("8-bit input slot not allocated");
    const int key = n * 4 + slot + (u8 ? 2 : 0);
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaGraph_t g;
        if (!e->cuda_ok(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal), "begin capture"))
            return PTQ8_ERR_CUDA;
        e->cur_input = slot ? e->d_input2 : e->d_input;
        e->cur_input_u8 = u8 ? e->d_input_u8[slot] : nullptr;
        int rc = enqueue(e, n);
        e->cur_input = nullptr;
        e->cur_input_u8 = nullptr;
        cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
        if (rc) return rc;
        if (!e->cuda_ok(ce, "end capture")) return PTQ8_ERR_CUDA;
        cudaGraphExec_t ge;
        ce = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (!e->cuda_ok(ce, "graph instantiate")) return PTQ8_ERR_CUDA;
        it = e->graphs.emplace(key, ge).first;
    }
    *out = it->second;
    return PTQ8_OK;
}

int launch(ptq8_engine* e, int n, bool use_graph) {
    if (!use_graph) {
        if (!e->planned) {
            int rc = finalize(e, std::max(n, e->max_batch > 0 ? e->max_batch : n));
            if (rc) return rc;
        }
        if (n <= 0 || n > e->max_batch)
            return e->fail(strf("batch %d outside [1, %d] (alloc_scratch sets the maximum)", n, e->max_batch));
        if (!e->cuda_ok(cudaSetDevice(e->device), "cudaSetDevice")) return PTQ8_ERR_CUDA;
        return enqueue(e, n);
    }
    cudaGraphExec_t ge;
    int rc = graph_for(e, n, &ge);
    if (rc) return rc;
    if (!e->cuda_ok(cudaGraphLaunch(ge, e->stream), "graph launch")) return PTQ8_ERR_CUDA;
    return PTQ8_OK;
}

// Work just enqueued on the engine stream reads input slot 0 (d_input): a pipelined
// forward must not overwrite that slot before it has run, so the slot's "free" event
// moves past it (once the pipelined path exists; until then nothing copies into the
// slot from another stream).
void mark_input_read(ptq8_engine* e) {
    if (e->ev_free[0]) cudaEventRecord(e->ev_free[0], e->stream);
}

// A PTQC-style range the device quantizer accepts: the rules ptq8_engine_set_calib
// and load_ptqc enforce (finite, lo <= hi; ptq_model.h:425-503), a known scale mode,
// and a finite positive scale (the precondition of make_qparams).
bool quant_range_ok(float lo, float hi, int mode, std::string& why) {
    if (mode != ACT_ABSMAX && mode != ACT_MINMAX) {
        why = strf("act mode %d: must be %d (absmax) or %d (minmax)", mode, (int)ACT_ABSMAX, (int)ACT_MINMAX);
        return false;
    }
    if (!std::isfinite(lo) || !std::isfinite(hi)) {
        why = "calibration range not finite";
        return false;
    }
    if (lo > hi) {
        why = "calibration range lo > hi";
        return false;
    }
    if (!qparams_scale_ok(act_scale_from_range(lo, hi, 8, mode))) {
        why = "activation scale not finite and positive";
        return false;
    }
    return true;
}

void copy_err(const std::string& m, char* err, size_t errlen) {
    if (err && errlen) {
        std::snprintf(err, errlen, "%s", m.c_str());
    }
}

}  // namespace

// ---------------------------------------------------------------- fixed scratch
// Device memory of ptq8_quantize_device_noalloc, part of the loaded module (one
// copy per device), so the call never allocates: PTQ8_NOALLOC_MAX_VALUES float
// inputs, then as many code bytes.  Every call on a device reuses the same bytes
// and leaves its own data behind; nothing here has to start at zero because the
// call reads back only the codes its kernel has just written.
constexpr size_t kNoAllocCodesOff = static_cast<size_t>(PTQ8_NOALLOC_MAX_VALUES) * 4;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocCodesOff + PTQ8_NOALLOC_MAX_VALUES];

namespace {

// Device address of g_noalloc_scratch on the current device.  Looked up on every
// call (the lookup allocates nothing): a remembered address would go stale when the
// device's primary context is reset and the module reloaded.
unsigned char* noalloc_scratch(std::string& why) {
    void* p = nullptr;
    const cudaError_t ce = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (ce != cudaSuccess || !p) {
        why = strf("cudaGetSymbolAddress of the fixed scratch failed: %s", cudaGetErrorString(ce));
        return nullptr;
    }
    return static_cast<unsigned char*>(p);
}

}  // namespace

// ====================================================================== C ABI

extern "C" {

int ptq8_abi_version(void) { return PTQ8_ABI_VERSION; }

ptq8_model* ptq8_model_load(const char* path, char* err, size_t errlen) {
    try {
        if (!path) {
            copy_err("null path", err, errlen);
            return nullptr;
        }
        std::unique_ptr<ptq8_model> m(new ptq8_model());
        std::string e;
        if (!m->m.load(path, &e)) {
            copy_err(e, err, errlen);
            return nullptr;
        }
        copy_err("", err, errlen);
        return m.release();
    } catch (const std::exception& ex) {
        copy_err(std::string("ptq8_model_load: ") + ex.what(), err, errlen);
        return nullptr;
    }
}

void ptq8_model_free(ptq8_model* m) { delete m; }

int ptq8_model_info(const ptq8_model* mm, int* out) {
    if (!mm || !out) return PTQ8_ERR_INVALID;
    const Model& m = mm->m;
    int n_dw = 0, n_grouped = 0, n_relu6 = 0, n_res2 = 0;
    for (const ConvSpec& c : m.convs) {
        n_dw += c.depthwise();
        n_grouped += c.groups != 1;
        n_relu6 += c.relu == 2;
    }
    for (const BlockSpec& b : m.blocks) n_res2 += b.residual == 2;
    out[0] = (int)m.convs.size();
    out[1] = (int)m.blocks.size();
    out[2] = m.stem_pool;
    out[3] = m.fc_in;
    out[4] = m.fc_out;
    out[5] = n_dw;
    out[6] = n_grouped;
    out[7] = n_relu6;
    out[8] = n_res2;
    out[9] = m.magic == "PTQ8" ? 3 : (m.magic == "PTQ2" ? 2 : 1);
    out[10] = m.blocks.empty() ? 0 : (int)m.blocks[0].convs.size();
    return PTQ8_OK;
}

int ptq8_model_conv(const ptq8_model* mm, int i, int* meta10) {
    if (!mm || !meta10 || i < 0 || i >= (int)mm->m.convs.size()) return PTQ8_ERR_INVALID;
    const ConvSpec& c = mm->m.convs[i];
    const int v[10] = {c.cout, c.cin, c.kh, c.kw, c.sh, c.sw, c.ph, c.pw, c.relu, c.groups};
    std::memcpy(meta10, v, sizeof v);
    return PTQ8_OK;
}

int ptq8_model_block(const ptq8_model* mm, int i, int* convs, int cap, int* n_convs, int* ds, int* stride,
                     int* residual) {
    if (!mm || i < 0 || i >= (int)mm->m.blocks.size()) return PTQ8_ERR_INVALID;
    const BlockSpec& b = mm->m.blocks[i];
    if (n_convs) *n_convs = (int)b.convs.size();
    for (int k = 0; k < (int)b.convs.size() && k < cap && convs; ++k) convs[k] = b.convs[k];
    if (ds) *ds = b.ds;
    if (stride) *stride = b.stride;
    if (residual) *residual = b.residual;
    return PTQ8_OK;
}

int ptq8_model_weights(const ptq8_model* mm, int i, const float** weight, size_t* n_weight, const float** bias) {
    if (!mm || i < -1 || i >= (int)mm->m.convs.size()) return PTQ8_ERR_INVALID;
    if (i == -1) {
        if (weight) *weight = mm->m.fc_w.data();
        if (n_weight) *n_weight = mm->m.fc_w.size();
        if (bias) *bias = mm->m.fc_b.data();
        return PTQ8_OK;
    }
    const ConvSpec& c = mm->m.convs[i];
    if (weight) *weight = c.weight.data();
    if (n_weight) *n_weight = c.weight.size();
    if (bias) *bias = c.bias.data();
    return PTQ8_OK;
}

int ptq8_model_codes(const ptq8_model* mm, int i, const int8_t** codes, size_t* n_codes, const float** scales,
                     int* bits) {
    if (!mm || i < 0 || i >= (int)mm->m.convs.size()) return PTQ8_ERR_INVALID;
    const ConvSpec& c = mm->m.convs[i];
    if (codes) *codes = c.codes.empty() ? nullptr : c.codes.data();
    if (n_codes) *n_codes = c.codes.size();
    if (scales) *scales = c.wscale.empty() ? nullptr : c.wscale.data();
    if (bits) *bits = c.qbits;
    return PTQ8_OK;
}

int ptq8_load_ptqc(const char* path, size_t n_expected, float* lohi, size_t cap, char* err, size_t errlen) {
    try {
        if (!path) {
            copy_err("null path", err, errlen);
            return PTQ8_ERR_INVALID;
        }
        std::vector<std::pair<float, float>> r;
        std::string e;
        if (!load_ptqc(path, n_expected, &r, &e)) {
            copy_err(e, err, errlen);
            return PTQ8_ERR_FORMAT;
        }
        if (lohi) {
            if (cap < 2 * r.size()) {
                copy_err("output buffer too small", err, errlen);
                return PTQ8_ERR_INVALID;
            }
            for (size_t k = 0; k < r.size(); ++k) {
                lohi[2 * k] = r[k].first;
                lohi[2 * k + 1] = r[k].second;
            }
        }
        copy_err("", err, errlen);
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        copy_err(std::string("ptq8_load_ptqc: ") + ex.what(), err, errlen);
        return PTQ8_ERR_FORMAT;
    }
}

double ptq8_act_scale(float lo, float hi, int bits, int mode) { return act_scale_from_range(lo, hi, bits, mode); }

int ptq8_quantize_weight(const float* w, int cout, int k, int bits, int8_t* codes, float* scale32) {
    if (!w || !codes || !scale32 || cout <= 0 || k <= 0 || bits < 2 || bits > 8) return PTQ8_ERR_INVALID;
    quantize_weight_per_channel(w, cout, k, bits, codes, scale32);
    return PTQ8_OK;
}

int ptq8_quantize_device(int device, const float* x_host, size_t n, float lo, float hi, int mode, int8_t* codes) {
    if (!x_host || !codes) return PTQ8_ERR_INVALID;
    std::string why;
    if (!quant_range_ok(lo, hi, mode, why)) return PTQ8_ERR_INVALID;
    if (cudaSetDevice(device) != cudaSuccess) return PTQ8_ERR_CUDA;
    const double s = act_scale_from_range(lo, hi, 8, mode);
    float* dx = nullptr;
    int8_t* dq = nullptr;
    const size_t nn = n ? n : 1;
    if (cudaMalloc(&dx, nn * 4) != cudaSuccess) return PTQ8_ERR_CUDA;
    if (cudaMalloc(&dq, nn + 32) != cudaSuccess) {
        cudaFree(dx);
        return PTQ8_ERR_CUDA;
    }
    int rc = PTQ8_OK;
    if (cudaMemcpy(dx, x_host, n * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = PTQ8_ERR_CUDA;
    if (!rc && n) {
        const size_t groups = (n + 15) / 16;
        quantize_kernel<<<(unsigned)((groups + 127) / 128), 128>>>(dx, n, make_qparams(s), (float)(1.0 / s), s, dq);
        if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) rc = PTQ8_ERR_CUDA;
    }
    if (!rc && cudaMemcpy(codes, dq, n, cudaMemcpyDeviceToHost) != cudaSuccess) rc = PTQ8_ERR_CUDA;
    cudaFree(dx);
    cudaFree(dq);
    return rc;
}

int ptq8_quantize_device_noalloc(int device, const float* x_host, size_t n, float lo, float hi, int mode,
                                 int8_t* codes, char* err, size_t errlen) {
    if (!x_host || !codes) {
        copy_err("null input or output pointer", err, errlen);
        return PTQ8_ERR_INVALID;
    }
    if (device < 0) {
        copy_err(strf("device %d is negative", device), err, errlen);
        return PTQ8_ERR_INVALID;
    }
    std::string bad;
    if (!quant_range_ok(lo, hi, mode, bad)) {
        copy_err(bad, err, errlen);
        return PTQ8_ERR_INVALID;
    }
    if (n > static_cast<size_t>(PTQ8_NOALLOC_MAX_VALUES)) {
        copy_err(strf("n = %zu exceeds the fixed scratch of %u values; split the call or use ptq8_quantize_device",
                      n, static_cast<unsigned>(PTQ8_NOALLOC_MAX_VALUES)),
                 err, errlen);
        return PTQ8_ERR_INVALID;
    }
    cudaError_t ce = cudaSetDevice(device);
    if (ce != cudaSuccess) {
        copy_err(strf("cudaSetDevice(%d): %s", device, cudaGetErrorString(ce)), err, errlen);
        return PTQ8_ERR_CUDA;
    }
    std::string why;
    unsigned char* base = noalloc_scratch(why);
    if (!base) {
        copy_err(why, err, errlen);
        return PTQ8_ERR_CUDA;
    }
    if (n == 0) {
        copy_err("", err, errlen);
        return PTQ8_OK;
    }
    float* dx = reinterpret_cast<float*>(base);
    int8_t* dq = reinterpret_cast<int8_t*>(base + kNoAllocCodesOff);
    const double s = act_scale_from_range(lo, hi, 8, mode);
    // Legacy default stream throughout: the device-to-host copy is ordered after the kernel.
    ce = cudaMemcpy(dx, x_host, n * 4, cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) {
        const size_t groups = (n + 15) / 16;
        quantize_kernel<<<(unsigned)((groups + 127) / 128), 128>>>(dx, n, make_qparams(s), (float)(1.0 / s), s, dq);
        ce = cudaGetLastError();
    }
    if (ce == cudaSuccess) ce = cudaMemcpy(codes, dq, n, cudaMemcpyDeviceToHost);
    if (ce != cudaSuccess) {
        copy_err(strf("CUDA: %s", cudaGetErrorString(ce)), err, errlen);
        return PTQ8_ERR_CUDA;
    }
    copy_err("", err, errlen);
    return PTQ8_OK;
}

ptq8_engine* ptq8_engine_create(int device) {
    auto* e = new ptq8_engine();
    e->device = device;
    return e;
}

void ptq8_engine_destroy(ptq8_engine* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    delete e;
}

const char* ptq8_engine_last_error(const ptq8_engine* e) { return e ? e->err.c_str() : "null engine"; }

int ptq8_engine_build(ptq8_engine* e, const ptq8_model* mm, int w_bits, int a_bits, const int* layer_bits,
                      int n_layer_bits, int passes) {
    try {
        if (!e || !mm) return PTQ8_ERR_INVALID;
        const Model& m = mm->m;
        if (a_bits != 8) return e->fail(strf("a_bits=%d unsupported (int8 activations only)", a_bits));
        if (w_bits != 8 && w_bits != 4) return e->fail(strf("w_bits=%d unsupported (8 or 4)", w_bits));
        if (layer_bits && n_layer_bits != (int)m.convs.size())
            return e->fail(strf("layer plan has %d entries but the model has %zu convs", n_layer_bits, m.convs.size()));
        e->model = &m;
        e->w_bits = w_bits;
        e->a_bits = a_bits;
        e->passes = passes;
        e->layer_bits.assign(m.convs.size(), w_bits);
        if (layer_bits)
            for (size_t i = 0; i < m.convs.size(); ++i) {
                if (layer_bits[i] != 8 && layer_bits[i] != 4)
                    return e->fail(strf("layer plan: conv %zu bits=%d (4/8 only)", i, layer_bits[i]));
                e->layer_bits[i] = layer_bits[i];
            }
        // a PTQ8 package carries each conv's codes and bits: they rule (a plan must agree)
        for (size_t i = 0; i < m.convs.size(); ++i) {
            const int qb = m.convs[i].qbits;
            if (qb == 0) continue;
            if (layer_bits && layer_bits[i] != qb)
                return e->fail(strf("layer plan: conv %zu bits=%d but the package stores W%d codes", i, layer_bits[i], qb));
            e->layer_bits[i] = qb;
        }
        std::string verr;
        if (!m.validate(&verr, e->in_h, e->in_w)) return e->fail(verr);
        e->q.assign(m.convs.size(), ConvQ());
        for (size_t i = 0; i < m.convs.size(); ++i) {
            const ConvSpec& c = m.convs[i];
            ConvQ& cq = e->q[i];
            cq.spec = c;
            cq.spec.weight.clear();
            cq.spec.bias.clear();
            cq.spec.codes.clear();
            cq.spec.wscale.clear();
            cq.bits = e->layer_bits[i];
            const int K = c.cin * c.kh * c.kw;
            if (c.qbits > 0) {   // PTQ8: the stored codes and scales, no re-quantization
                cq.codes = c.codes;
                cq.wscale = c.wscale;
            } else {
                cq.codes.resize((size_t)c.cout * K);
                cq.wscale.resize(c.cout);
                quantize_weight_per_channel(c.weight.data(), c.cout, K, cq.bits, cq.codes.data(), cq.wscale.data());
            }
            cq.bias = c.bias;
        }
        // graph passes run on the quantized layers (codes + scales), so they are exact
        e->passes_log.clear();
        if (passes) {
            int h = conv_out_dim(e->in_h, m.convs[0].kh, m.convs[0].sh, m.convs[0].ph);
            int w = conv_out_dim(e->in_w, m.convs[0].kw, m.convs[0].sw, m.convs[0].pw);
            if (m.stem_pool) { h = (h + 2 - 3) / 2 + 1; w = (w + 2 - 3) / 2 + 1; }
            for (size_t bi = 0; bi < m.blocks.size(); ++bi) {
                const BlockSpec& b = m.blocks[bi];
                auto try_conv = [&](int ci, int ih, int iw) {
                    std::string note;
                    bool done = false;
                    if (passes & PTQ8_PASS_CENTER_TAP) done = center_tap(e->q[ci], ih, iw, &note);
                    if (!done && (passes & PTQ8_PASS_DECOMPOSE)) done = decompose(e->q[ci], ih, iw, &note);
                    if (!done && (passes & PTQ8_PASS_POSITIONAL)) done = positional(e->q[ci], ih, iw, &note);
                    e->passes_log.push_back(strf("conv[%d] in %dx%d: %s", ci, ih, iw, done ? note.c_str() : "unchanged"));
                };
                if (b.ds >= 0) try_conv(b.ds, h, w);
                int th = h, tw = w;
                for (int ci : b.convs) {
                    if (ci < 0) continue;
                    const ConvSpec& c = m.convs[ci];
                    try_conv(ci, th, tw);
                    th = conv_out_dim(th, c.kh, c.sh, c.ph);
                    tw = conv_out_dim(tw, c.kw, c.sw, c.pw);
                }
                h = th;
                w = tw;
            }
        }
        e->built = true;
        e->planned = false;
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        return e->fail(std::string("build: ") + ex.what());
    }
}

int ptq8_engine_set_act_mode(ptq8_engine* e, int mode) {
    if (!e) return PTQ8_ERR_INVALID;
    if (mode != ACT_ABSMAX && mode != ACT_MINMAX) return e->fail("act mode must be 0 (absmax) or 1 (minmax)");
    e->act_mode = mode;
    if (e->calibrated) {
        for (size_t i = 0; i < e->ranges.size(); ++i)
            e->scale[i] = act_scale_from_range(e->ranges[i].first, e->ranges[i].second, e->a_bits, e->act_mode);
        e->planned = false;
    }
    return PTQ8_OK;
}

int ptq8_engine_set_calib(ptq8_engine* e, const float* lohi, size_t n) {
    if (!e) return PTQ8_ERR_INVALID;
    if (!e->built) return e->fail("set_calib before build");
    if (n != e->q.size()) return e->fail(strf("calibration layer count %zu != conv count %zu", n, e->q.size()));
    std::vector<std::pair<float, float>> r(n);
    for (size_t i = 0; i < n; ++i) {
        const float lo = lohi[2 * i], hi = lohi[2 * i + 1];
        if (!std::isfinite(lo) || !std::isfinite(hi)) return e->fail(strf("layer %zu calibration range not finite", i));
        if (lo > hi) return e->fail(strf("layer %zu calibration range lo > hi", i));
        r[i] = {lo, hi};
    }
    e->ranges = r;
    e->scale.resize(n);
    for (size_t i = 0; i < n; ++i) e->scale[i] = act_scale_from_range(r[i].first, r[i].second, e->a_bits, e->act_mode);
    e->calibrated = true;
    e->planned = false;
    return PTQ8_OK;
}

int ptq8_engine_set_input_shape(ptq8_engine* e, int c, int h, int w) {
    if (!e || c <= 0 || h <= 0 || w <= 0) return PTQ8_ERR_INVALID;
    e->in_c = c;
    e->in_h = h;
    e->in_w = w;
    e->planned = false;
    return PTQ8_OK;
}

int ptq8_engine_alloc_scratch(ptq8_engine* e, int max_batch) {
    if (!e) return PTQ8_ERR_INVALID;
    return finalize(e, max_batch);
}

int ptq8_engine_set_max_ctas(ptq8_engine* e, int max_ctas) {
    if (!e || max_ctas < 0) return PTQ8_ERR_INVALID;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);   // captured with the old grids
    e->graphs.clear();
    e->max_ctas = max_ctas;
    return PTQ8_OK;
}

int ptq8_engine_set_stream(ptq8_engine* e, void* stream) {
    if (!e) return PTQ8_ERR_INVALID;
    // work still queued on the old stream (or input copies on the copy stream) uses the
    // activations, logits and input slots the new stream is about to reuse
    if (e->stream && !e->cuda_ok(cudaStreamSynchronize(e->stream), "sync old stream")) return PTQ8_ERR_CUDA;
    if (e->copy_stream && !e->cuda_ok(cudaStreamSynchronize(e->copy_stream), "sync copy stream")) return PTQ8_ERR_CUDA;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
    if (e->own_stream && e->stream) cudaStreamDestroy(e->stream);
    e->own_stream = false;
    e->stream = static_cast<cudaStream_t>(stream);
    if (!e->stream) {
        if (!e->cuda_ok(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream")) return PTQ8_ERR_CUDA;
        e->own_stream = true;
    }
    return PTQ8_OK;
}

void* ptq8_engine_stream(ptq8_engine* e) { return e ? static_cast<void*>(e->stream) : nullptr; }

float* ptq8_engine_input_buffer(ptq8_engine* e) {
    if (!e) return nullptr;
    // a pipelined call's copy into this buffer may still be in flight, and a forward
    // queued on the engine stream may still be reading it
    if (e->copy_stream) cudaStreamSynchronize(e->copy_stream);
    if (e->stream) cudaStreamSynchronize(e->stream);
    return e->d_input;
}
float* ptq8_engine_logits_buffer(ptq8_engine* e) { return e ? e->d_logits : nullptr; }

int ptq8_engine_run(ptq8_engine* e, int n, int use_graph) {
    if (!e) return PTQ8_ERR_INVALID;
    if (e->copy_stream && !e->cuda_ok(cudaStreamSynchronize(e->copy_stream), "copy stream")) return PTQ8_ERR_CUDA;
    const int rc = launch(e, n, use_graph != 0);
    if (!rc) mark_input_read(e);
    return rc;
}

int ptq8_engine_forward_device(ptq8_engine* e, const float* x_dev, int n, float* logits_dev) {
    if (!e || !x_dev || !logits_dev) return PTQ8_ERR_INVALID;
    if (!e->planned) {
        int rc = finalize(e, std::max(n, e->max_batch));
        if (rc) return rc;
    }
    if (n <= 0 || n > e->max_batch) return e->fail(strf("batch %d outside [1, %d]", n, e->max_batch));
    if (e->copy_stream && !e->cuda_ok(cudaStreamSynchronize(e->copy_stream), "copy stream")) return PTQ8_ERR_CUDA;
    const size_t in_bytes = (size_t)n * e->in_c * e->in_h * e->in_w * sizeof(float);
    if (x_dev != e->d_input &&
        !e->cuda_ok(cudaMemcpyAsync(e->d_input, x_dev, in_bytes, cudaMemcpyDeviceToDevice, e->stream), "input copy"))
        return PTQ8_ERR_CUDA;
    int rc = launch(e, n, true);
    if (rc) return rc;
    mark_input_read(e);
    if (logits_dev != e->d_logits &&
        !e->cuda_ok(cudaMemcpyAsync(logits_dev, e->d_logits, (size_t)n * e->model->fc_out * sizeof(float),
                                    cudaMemcpyDeviceToDevice, e->stream),
                    "logits copy"))
        return PTQ8_ERR_CUDA;
    return PTQ8_OK;
}

int ptq8_engine_forward(ptq8_engine* e, const float* x_host, int n, int c, int h, int w, float* logits_host) {
    if (!e || !x_host || !logits_host) return PTQ8_ERR_INVALID;
    if (c != e->in_c || h != e->in_h || w != e->in_w)
        return e->fail(strf("input shape %dx%dx%d != engine input %dx%dx%d", c, h, w, e->in_c, e->in_h, e->in_w));
    if (!e->planned) {
        int rc = finalize(e, std::max(n, e->max_batch));
        if (rc) return rc;
    }
    if (n <= 0 || n > e->max_batch) return e->fail(strf("batch %d outside [1, %d]", n, e->max_batch));
    // a pipelined call's copy into the same input slot may still be in flight
    if (e->copy_stream && !e->cuda_ok(cudaStreamSynchronize(e->copy_stream), "copy stream")) return PTQ8_ERR_CUDA;
    const size_t in_bytes = (size_t)n * c * h * w * sizeof(float);
    if (!e->cuda_ok(cudaMemcpyAsync(e->d_input, x_host, in_bytes, cudaMemcpyHostToDevice, e->stream), "H2D"))
        return PTQ8_ERR_CUDA;
    int rc = launch(e, n, true);
    if (rc) return rc;
    mark_input_read(e);
    if (!e->cuda_ok(cudaMemcpyAsync(logits_host, e->d_logits, (size_t)n * e->model->fc_out * sizeof(float),
                                    cudaMemcpyDeviceToHost, e->stream),
                    "D2H"))
        return PTQ8_ERR_CUDA;
    if (!e->cuda_ok(cudaStreamSynchronize(e->stream), "forward")) return PTQ8_ERR_CUDA;
    return ptq8_engine_check_device_error(e);
}

namespace {

// The pipelined forwards' copy stream and per-slot events, created on first use.
int ensure_copy_stream(ptq8_engine* e) {
    if (e->copy_stream) return PTQ8_OK;
    if (!e->cuda_ok(cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking), "copy stream"))
        return PTQ8_ERR_CUDA;
    for (int k = 0; k < 2; ++k)
        if (!e->cuda_ok(cudaEventCreateWithFlags(&e->ev_staged[k], cudaEventDisableTiming), "event") ||
            !e->cuda_ok(cudaEventCreateWithFlags(&e->ev_free[k], cudaEventDisableTiming), "event") ||
            // work already queued on the engine stream (a forward_device or run graph
            // reading slot 0) must finish before the first pipelined copy overwrites a slot
            !e->cuda_ok(cudaEventRecord(e->ev_free[k], e->stream), "record free"))
            return PTQ8_ERR_CUDA;
    return PTQ8_OK;
}

}  // namespace

int ptq8_engine_forward_async(ptq8_engine* e, const float* x_host, int n, float* logits_host) {
    try {
        if (!e || !x_host || !logits_host) return PTQ8_ERR_INVALID;
        if (!e->planned) {
            int rc = finalize(e, std::max(n, e->max_batch));
            if (rc) return rc;
        }
        if (n <= 0 || n > e->max_batch) return e->fail(strf("batch %d outside [1, %d]", n, e->max_batch));
        if (!e->cuda_ok(cudaSetDevice(e->device), "cudaSetDevice")) return PTQ8_ERR_CUDA;
        const size_t in_bytes = (size_t)n * e->in_c * e->in_h * e->in_w * sizeof(float);
        int rc = ensure_copy_stream(e);
        if (rc) return rc;
        if (!e->d_input2 &&
            !e->dalloc(&e->d_input2, (size_t)e->max_batch * e->in_c * e->in_h * e->in_w * sizeof(float),
                       "alloc second input slot"))
            return PTQ8_ERR_CUDA;
        const int slot = e->async_slot;
        float* dst = slot ? e->d_input2 : e->d_input;
        cudaGraphExec_t ge;
        rc = graph_for(e, n, &ge, slot);
        if (rc) return rc;
        // the slot is free once the forward that last read it has run (a never-recorded
        // event is no dependency)
        if (!e->cuda_ok(cudaStreamWaitEvent(e->copy_stream, e->ev_free[slot], 0), "wait slot") ||
            !e->cuda_ok(cudaMemcpyAsync(dst, x_host, in_bytes, cudaMemcpyHostToDevice, e->copy_stream), "H2D") ||
            !e->cuda_ok(cudaEventRecord(e->ev_staged[slot], e->copy_stream), "record staged") ||
            !e->cuda_ok(cudaStreamWaitEvent(e->stream, e->ev_staged[slot], 0), "wait staged") ||
            !e->cuda_ok(cudaGraphLaunch(ge, e->stream), "graph launch") ||
            !e->cuda_ok(cudaEventRecord(e->ev_free[slot], e->stream), "record free") ||
            !e->cuda_ok(cudaMemcpyAsync(logits_host, e->d_logits, (size_t)n * e->model->fc_out * sizeof(float),
                                        cudaMemcpyDeviceToHost, e->stream),
                        "D2H"))
            return PTQ8_ERR_CUDA;
        e->async_slot ^= 1;
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        return e ? e->fail(strf("forward_async: %s", ex.what()), PTQ8_ERR_CUDA) : PTQ8_ERR_CUDA;
    }
}

int ptq8_engine_set_input_norm(ptq8_engine* e, int mode, const float* mean, const float* std_) {
    if (!e) return PTQ8_ERR_INVALID;
    if (mode != PTQ8_NORM_DIV && mode != PTQ8_NORM_MUL)
        return e->fail(strf("input normalisation mode %d: must be %d (div) or %d (mul)", mode, PTQ8_NORM_DIV,
                            PTQ8_NORM_MUL));
    if ((mean == nullptr) != (std_ == nullptr)) return e->fail("mean and std: both given or both NULL");
    if (e->in_c > 4) return e->fail(strf("8-bit input: at most 4 channels (engine input has %d)", e->in_c));
    U8Norm nm;
    if (!mean) {
        if (e->in_c != 3) return e->fail("the CIFAR-10 constants need a 3-channel input");
        nm = cifar_norm(mode);
    } else {
        for (int k = 0; k < e->in_c; ++k)
            if (!std::isfinite(mean[k]) || !std::isfinite(std_[k]) || !(std_[k] > 0.0f))
                return e->fail(strf("channel %d: mean must be finite and std finite and positive", k));
        nm = make_norm(mode, mean, std_, e->in_c);
        for (int k = 0; k < e->in_c; ++k)
            if (!std::isfinite(nm.m[k]) || !std::isfinite(nm.d[k]) || !(nm.d[k] > 0.0f))
                return e->fail(strf("channel %d: normalisation constants overflow float32", k));
    }
    // graphs of 8-bit forwards carry the constants as kernel parameters
    if (e->stream && !e->cuda_ok(cudaStreamSynchronize(e->stream), "sync")) return PTQ8_ERR_CUDA;
    for (auto it = e->graphs.begin(); it != e->graphs.end();) {
        if (it->first & 2) {
            cudaGraphExecDestroy(it->second);
            it = e->graphs.erase(it);
        } else {
            ++it;
        }
    }
    e->u8_norm = nm;
    return PTQ8_OK;
}

namespace {

// Checks shared by the 8-bit input forwards; allocates 8-bit input slot `slot` on first use.
int u8_prepare(ptq8_engine* e, int n, size_t record_bytes, int slot, size_t* img_bytes) {
    if (!e->planned) {
        int rc = finalize(e, std::max(n, e->max_batch));
        if (rc) return rc;
    }
    if (n <= 0 || n > e->max_batch) return e->fail(strf("batch %d outside [1, %d]", n, e->max_batch));
    if (e->in_c > 4) return e->fail(strf("8-bit input: at most 4 channels (engine input has %d)", e->in_c));
    *img_bytes = (size_t)e->in_c * e->in_h * e->in_w;
    if (record_bytes != 0 && record_bytes < *img_bytes)
        return e->fail(strf("record_bytes %zu < %zu pixel bytes per image", record_bytes, *img_bytes));
    if (!e->cuda_ok(cudaSetDevice(e->device), "cudaSetDevice")) return PTQ8_ERR_CUDA;
    if (!e->d_input_u8[slot] && !e->dalloc(&e->d_input_u8[slot], (size_t)e->max_batch * *img_bytes, "alloc 8-bit input"))
        return PTQ8_ERR_CUDA;
    return PTQ8_OK;
}

// Copy of n images of img_bytes pixels, record_bytes apart at src (0: packed), into a packed slot.
cudaError_t copy_records(uint8_t* dst, const uint8_t* src, int n, size_t img_bytes, size_t record_bytes,
                         cudaMemcpyKind kind, cudaStream_t s) {
    if (record_bytes == 0 || record_bytes == img_bytes)
        return cudaMemcpyAsync(dst, src, (size_t)n * img_bytes, kind, s);
    return cudaMemcpy2DAsync(dst, img_bytes, src, record_bytes, img_bytes, n, kind, s);
}

}  // namespace

int ptq8_engine_forward_u8(ptq8_engine* e, const uint8_t* x_host, int n, size_t record_bytes, float* logits_host) {
    try {
        if (!e || !x_host || !logits_host) return PTQ8_ERR_INVALID;
        size_t img = 0;
        int rc = u8_prepare(e, n, record_bytes, 0, &img);
        if (rc) return rc;
        // a pipelined call's copy into the same slot may still be in flight
        if (e->copy_stream && !e->cuda_ok(cudaStreamSynchronize(e->copy_stream), "copy stream")) return PTQ8_ERR_CUDA;
        cudaGraphExec_t ge;
        if ((rc = graph_for(e, n, &ge, 0, true)) != 0) return rc;
        if (!e->cuda_ok(copy_records(e->d_input_u8[0], x_host, n, img, record_bytes, cudaMemcpyHostToDevice, e->stream),
                        "H2D") ||
            !e->cuda_ok(cudaGraphLaunch(ge, e->stream), "graph launch"))
            return PTQ8_ERR_CUDA;
        mark_input_read(e);
        if (!e->cuda_ok(cudaMemcpyAsync(logits_host, e->d_logits, (size_t)n * e->model->fc_out * sizeof(float),
                                        cudaMemcpyDeviceToHost, e->stream),
                        "D2H") ||
            !e->cuda_ok(cudaStreamSynchronize(e->stream), "forward"))
            return PTQ8_ERR_CUDA;
        return ptq8_engine_check_device_error(e);
    } catch (const std::exception& ex) {
        return e ? e->fail(strf("forward_u8: %s", ex.what()), PTQ8_ERR_CUDA) : PTQ8_ERR_CUDA;
    }
}

int ptq8_engine_forward_u8_async(ptq8_engine* e, const uint8_t* x_host, int n, size_t record_bytes,
                                 float* logits_host) {
    try {
        if (!e || !x_host || !logits_host) return PTQ8_ERR_INVALID;
        const int slot = e->async_slot;
        size_t img = 0;
        int rc = u8_prepare(e, n, record_bytes, slot, &img);
        if (rc) return rc;
        if ((rc = ensure_copy_stream(e)) != 0) return rc;
        cudaGraphExec_t ge;
        if ((rc = graph_for(e, n, &ge, slot, true)) != 0) return rc;
        // slot index k's free event follows the last forward that read either input of slot k
        if (!e->cuda_ok(cudaStreamWaitEvent(e->copy_stream, e->ev_free[slot], 0), "wait slot") ||
            !e->cuda_ok(copy_records(e->d_input_u8[slot], x_host, n, img, record_bytes, cudaMemcpyHostToDevice,
                                     e->copy_stream),
                        "H2D") ||
            !e->cuda_ok(cudaEventRecord(e->ev_staged[slot], e->copy_stream), "record staged") ||
            !e->cuda_ok(cudaStreamWaitEvent(e->stream, e->ev_staged[slot], 0), "wait staged") ||
            !e->cuda_ok(cudaGraphLaunch(ge, e->stream), "graph launch") ||
            !e->cuda_ok(cudaEventRecord(e->ev_free[slot], e->stream), "record free") ||
            !e->cuda_ok(cudaMemcpyAsync(logits_host, e->d_logits, (size_t)n * e->model->fc_out * sizeof(float),
                                        cudaMemcpyDeviceToHost, e->stream),
                        "D2H"))
            return PTQ8_ERR_CUDA;
        e->async_slot ^= 1;
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        return e ? e->fail(strf("forward_u8_async: %s", ex.what()), PTQ8_ERR_CUDA) : PTQ8_ERR_CUDA;
    }
}

int ptq8_engine_forward_device_u8(ptq8_engine* e, const uint8_t* x_dev, int n, size_t record_bytes,
                                  float* logits_dev) {
    try {
        if (!e || !x_dev || !logits_dev) return PTQ8_ERR_INVALID;
        size_t img = 0;
        int rc = u8_prepare(e, n, record_bytes, 0, &img);
        if (rc) return rc;
        if (e->copy_stream && !e->cuda_ok(cudaStreamSynchronize(e->copy_stream), "copy stream")) return PTQ8_ERR_CUDA;
        cudaGraphExec_t ge;
        if ((rc = graph_for(e, n, &ge, 0, true)) != 0) return rc;
        if (!e->cuda_ok(copy_records(e->d_input_u8[0], x_dev, n, img, record_bytes, cudaMemcpyDeviceToDevice, e->stream),
                        "input copy") ||
            !e->cuda_ok(cudaGraphLaunch(ge, e->stream), "graph launch"))
            return PTQ8_ERR_CUDA;
        mark_input_read(e);
        if (logits_dev != e->d_logits &&
            !e->cuda_ok(cudaMemcpyAsync(logits_dev, e->d_logits, (size_t)n * e->model->fc_out * sizeof(float),
                                        cudaMemcpyDeviceToDevice, e->stream),
                        "logits copy"))
            return PTQ8_ERR_CUDA;
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        return e ? e->fail(strf("forward_device_u8: %s", ex.what()), PTQ8_ERR_CUDA) : PTQ8_ERR_CUDA;
    }
}

int ptq8_engine_copy_logits(ptq8_engine* e, int n, float* dst_dev) {
    if (!e || !dst_dev || !e->planned || n <= 0 || n > e->max_batch) return PTQ8_ERR_INVALID;
    if (!e->cuda_ok(cudaMemcpyAsync(dst_dev, e->d_logits, (size_t)n * e->model->fc_out * sizeof(float),
                                    cudaMemcpyDeviceToDevice, e->stream),
                    "logits copy"))
        return PTQ8_ERR_CUDA;
    return PTQ8_OK;
}

int ptq8_engine_sync(ptq8_engine* e) {
    if (!e) return PTQ8_ERR_INVALID;
    if (!e->cuda_ok(cudaStreamSynchronize(e->stream), "sync")) return PTQ8_ERR_CUDA;
    return ptq8_engine_check_device_error(e);
}

int ptq8_engine_check_device_error(ptq8_engine* e) {
    if (!e) return PTQ8_ERR_INVALID;
    if (!e->d_err) return PTQ8_OK;   // nothing has run yet
    int v = 0;
    // ordered after this engine's enqueued work (its stream is non-blocking)
    if (!e->cuda_ok(cudaMemcpyAsync(&v, e->d_err, sizeof(int), cudaMemcpyDeviceToHost, e->stream), "read device error") ||
        !e->cuda_ok(cudaStreamSynchronize(e->stream), "read device error"))
        return PTQ8_ERR_CUDA;
    if (v != 0) {
        if (!e->cuda_ok(cudaMemsetAsync(e->d_err, 0, sizeof(int), e->stream), "clear device error") ||
            !e->cuda_ok(cudaStreamSynchronize(e->stream), "clear device error"))
            return PTQ8_ERR_CUDA;
        return e->fail(strf("device wait timed out (code %d); results of this forward are invalid", v), PTQ8_ERR_TIMEOUT);
    }
    return PTQ8_OK;
}

int ptq8_engine_set_wait_test(ptq8_engine* e, long long wait_limit_cycles, int stall_first_load) {
    if (!e || wait_limit_cycles < 0) return PTQ8_ERR_INVALID;
    if (e->stream && !e->cuda_ok(cudaStreamSynchronize(e->stream), "sync")) return PTQ8_ERR_CUDA;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);   // captured with the old parameters
    e->graphs.clear();
    e->wait_limit = wait_limit_cycles > 0 ? wait_limit_cycles : kWaitLimitCycles;
    e->stall_first_load = stall_first_load ? 1 : 0;
    return PTQ8_OK;
}

int ptq8_engine_tensor_info(ptq8_engine* e, int what, int index, int* shape4) {
    // what 0: input codes of conv `index` -> (N_max, H, W, ld); what 1: final fp32 map (N_max, H, W, C)
    if (!e || !e->planned || !shape4) return PTQ8_ERR_INVALID;
    if (what == 0) {
        if (index < 0 || index >= (int)e->conv_step.size() || e->conv_step[index] < 0) return PTQ8_ERR_INVALID;
        const Step& st = e->steps[e->conv_step[index]];
        if (st.kind == K_STEM_IM2COL) {
            shape4[0] = e->max_batch; shape4[1] = st.oh; shape4[2] = st.ow; shape4[3] = st.kpad;
        } else {   // a fused downsample reads (and reports) the even positions only
            const Value& v = e->vals[st.in_val];
            const bool sub = v.is_sub(v.code_index(st.s_in));
            shape4[0] = e->max_batch;
            shape4[1] = sub ? v.sub_h() : v.h;
            shape4[2] = sub ? v.sub_w() : v.w;
            shape4[3] = v.ldq;
        }
        return PTQ8_OK;
    }
    if (what == 1) {
        const Value& v = e->vals[e->final_val];
        shape4[0] = e->max_batch; shape4[1] = v.h; shape4[2] = v.w; shape4[3] = v.c;
        return PTQ8_OK;
    }
    return PTQ8_ERR_INVALID;
}

int ptq8_engine_dump(ptq8_engine* e, int what, int index, int n, void* host_dst, size_t bytes) {
    return ptq8_engine_dump_range(e, what, index, 0, n, host_dst, bytes);
}

int ptq8_engine_dump_range(ptq8_engine* e, int what, int index, int n0, int n, void* host_dst, size_t bytes) {
    try {
        if (!e || !e->planned || !host_dst || n0 < 0 || n <= 0 || n > e->max_batch || n0 > e->max_batch - n)
            return PTQ8_ERR_INVALID;
        int shp[4];
        int rc = ptq8_engine_tensor_info(e, what, index, shp);
        if (rc) return rc;
        const size_t elem = what == 0 ? 1 : sizeof(float);
        const size_t need = (size_t)n * shp[1] * shp[2] * shp[3] * elem;
        if (bytes < need) return e->fail("dump buffer too small");
        if (!e->cuda_ok(cudaStreamSynchronize(e->stream), "sync")) return PTQ8_ERR_CUDA;
        if (what == 0) {
            const Step& st = e->steps[e->conv_step[index]];
            if (st.kind == K_STEM_IM2COL) {   // drop the border rows of the bordered im2col map
                const size_t row = (size_t)st.ow * st.kpad, prow = (size_t)(st.ow + 2) * st.kpad;
                for (int i = 0; i < n; ++i) {
                    const int8_t* s0 = st.d_im2col + ((size_t)(n0 + i) * (st.oh + 2) + 1) * prow + st.kpad;
                    int8_t* d0 = static_cast<int8_t*>(host_dst) + (size_t)i * st.oh * row;
                    if (!e->cuda_ok(cudaMemcpy2D(d0, row, s0, prow, row, st.oh, cudaMemcpyDeviceToHost), "dump"))
                        return PTQ8_ERR_CUDA;
                }
                return PTQ8_OK;
            }
            const Value& v = e->vals[st.in_val];
            const int k = v.code_index(st.s_in);
            const int8_t* src = v.codes[k];
            const int H = v.is_sub(k) ? v.sub_h() : v.h, W = v.is_sub(k) ? v.sub_w() : v.w;
            // drop the one-pixel border: per image, H rows of W*ld bytes out of (H+2) x (W+2)*ld
            const size_t row = (size_t)W * v.ldq, prow = (size_t)(W + 2) * v.ldq;
            for (int i = 0; i < n; ++i) {
                const int8_t* s0 = src + ((size_t)(n0 + i) * (H + 2) + 1) * prow + v.ldq;
                int8_t* d0 = static_cast<int8_t*>(host_dst) + (size_t)i * H * row;
                if (!e->cuda_ok(cudaMemcpy2D(d0, row, s0, prow, row, H, cudaMemcpyDeviceToHost), "dump"))
                    return PTQ8_ERR_CUDA;
            }
            return PTQ8_OK;
        }
        // the device map is in the f32_off layout (whole 32-position blocks of all channels,
        // or plain NHWC): copy the blocks covering positions [p0, p1), then reorder to NHWC
        const Value& fv = e->vals[e->final_val];
        const size_t hw = (size_t)shp[1] * shp[2];
        const size_t p0 = (size_t)n0 * hw, p1 = p0 + (size_t)n * hw;
        const size_t b0 = p0 & ~(size_t)31, b1 = (p1 + 31) & ~(size_t)31;
        std::vector<float> raw((b1 - b0) * fv.c);
        if (!e->cuda_ok(cudaMemcpy(raw.data(), fv.f32 + b0 * fv.c, raw.size() * sizeof(float), cudaMemcpyDeviceToHost),
                        "dump"))
            return PTQ8_ERR_CUDA;
        float* dst = static_cast<float*>(host_dst);
        for (size_t p = p0; p < p1; ++p)
            for (int c = 0; c < fv.c; ++c) dst[(p - p0) * fv.c + c] = raw[f32_off(p - b0, c, fv.c)];
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        return e->fail(std::string("dump: ") + ex.what());
    }
}

int ptq8_engine_profile(ptq8_engine* e, int n, int iters, float* ms, double* macs, double* bytes, int* kind,
                        int cap, int* n_steps) {
    if (!e || iters <= 0) return PTQ8_ERR_INVALID;
    if (!e->planned) {
        int rc = finalize(e, std::max(n, e->max_batch));
        if (rc) return rc;
    }
    if (n <= 0 || n > e->max_batch) return e->fail("profile: batch outside the allocated range");
    if (e->copy_stream && !e->cuda_ok(cudaStreamSynchronize(e->copy_stream), "copy stream")) return PTQ8_ERR_CUDA;
    const int ns = (int)e->steps.size() + 1;
    if (n_steps) *n_steps = ns;
    if (cap < ns) return e->fail(strf("profile: needs %d entries", ns));
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    for (int si = 0; si < ns; ++si) {
        enqueue_step(e, n, si);   // warm
        cudaEventRecord(a, e->stream);
        for (int it = 0; it < iters; ++it) enqueue_step(e, n, si);
        cudaEventRecord(b, e->stream);
        if (!e->cuda_ok(cudaEventSynchronize(b), "profile")) {
            cudaEventDestroy(a);
            cudaEventDestroy(b);
            return PTQ8_ERR_CUDA;
        }
        float t = 0;
        cudaEventElapsedTime(&t, a, b);
        if (ms) ms[si] = t / iters;
        double mc, by;
        int k;
        step_work(e, n, si, &mc, &by, &k);
        if (macs) macs[si] = mc;
        if (bytes) bytes[si] = by;
        if (kind) kind[si] = k;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return ptq8_engine_check_device_error(e);
}

int ptq8_engine_weight_bytes(const ptq8_engine* e, size_t* device_bytes, size_t* int8_bytes, int* packed_convs) {
    if (!e || !e->planned) return PTQ8_ERR_INVALID;
    size_t dev = 0, i8 = 0;
    int np = 0;
    for (const Step& st : e->steps) {
        if (st.kind == K_MAXPOOL) continue;
        dev += st.w_dev_bytes;
        i8 += st.w_packed ? 2 * st.w_dev_bytes : st.w_dev_bytes;
        np += st.w_packed ? 1 : 0;
    }
    if (device_bytes) *device_bytes = dev;
    if (int8_bytes) *int8_bytes = i8;
    if (packed_convs) *packed_convs = np;
    return PTQ8_OK;
}

int ptq8_engine_n_launches(const ptq8_engine* e) {
    if (!e || !e->planned) return -1;
    int k = 1;   // head
    for (const Step& st : e->steps) k += st.fused ? 0 : st.kind == K_STEM_IM2COL ? 2 : 1;
    return k;
}

int ptq8_engine_passes_log(const ptq8_engine* e, char* out, size_t cap) {
    if (!e || !out || !cap) return PTQ8_ERR_INVALID;
    std::string s;
    for (const std::string& l : e->passes_log) s += l + "\n";
    std::snprintf(out, cap, "%s", s.c_str());
    return PTQ8_OK;
}

// ---- one-call interface (load / forward / debug / capture / destroy)

int ptq8_load(const char* model_path, const char* calib_path, const char* plan_json, const ptq8_opts* opts,
              ptq8_engine** out, char* err, size_t errlen) {
    try {
        if (out) *out = nullptr;
        if (!model_path || !calib_path || !out) {
            copy_err("null model path, calibration path or output pointer", err, errlen);
            return PTQ8_ERR_INVALID;
        }
        const ptq8_opts o = opts ? *opts : ptq8_opts{0, 8, 8, PTQ8_ACT_ABSMAX, 0, 0};
        ptq8_model* m = ptq8_model_load(model_path, err, errlen);
        if (!m) return PTQ8_ERR_FORMAT;
        const size_t nconv = m->m.convs.size();
        std::vector<float> lohi(2 * nconv);
        int rc = ptq8_load_ptqc(calib_path, nconv, lohi.data(), lohi.size(), err, errlen);
        if (rc) {
            ptq8_model_free(m);
            return rc;
        }
        std::vector<int> bits;
        std::string why;
        if (plan_json && !load_layer_plan(plan_json, nconv, &bits, &why)) {
            copy_err(why, err, errlen);
            ptq8_model_free(m);
            return PTQ8_ERR_FORMAT;
        }
        ptq8_engine* e = ptq8_engine_create(o.device);
        e->owned_model = m;
        rc = ptq8_engine_build(e, m, o.w_bits, o.a_bits, bits.empty() ? nullptr : bits.data(), (int)bits.size(),
                               o.passes);
        if (!rc) rc = ptq8_engine_set_act_mode(e, o.act_mode);
        if (!rc) rc = ptq8_engine_set_calib(e, lohi.data(), nconv);
        if (!rc && o.max_batch > 0) rc = ptq8_engine_alloc_scratch(e, o.max_batch);
        if (rc) {
            copy_err(e->err.empty() ? std::string("engine set-up failed") : e->err, err, errlen);
            ptq8_destroy(e);
            return rc;
        }
        copy_err("", err, errlen);
        *out = e;
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        copy_err(std::string("ptq8_load: ") + ex.what(), err, errlen);
        return PTQ8_ERR_INVALID;
    }
}

int ptq8_forward(ptq8_engine* e, const float* x_dev, int n, float* logits_dev, void* stream) {
    if (!e) return PTQ8_ERR_INVALID;
    if (stream && static_cast<cudaStream_t>(stream) != e->stream) {
        const int rc = ptq8_engine_set_stream(e, stream);
        if (rc) return rc;
    }
    return ptq8_engine_forward_device(e, x_dev, n, logits_dev);
}

int ptq8_forward_debug(ptq8_engine* e, const float* x_dev, int n, float* logits_dev, void* stream,
                       ptq8_dump_fn dump, void* user) {
    try {
        if (!e || !dump) return PTQ8_ERR_INVALID;
        int rc = ptq8_forward(e, x_dev, n, logits_dev, stream);
        if (rc) return rc;
        if ((rc = ptq8_engine_sync(e)) != 0) return rc;
        std::vector<int8_t> buf;
        for (int i = 0; i < (int)e->conv_step.size(); ++i) {
            if (e->conv_step[i] < 0) continue;   // conv folded away by a graph pass
            int shp[4];
            if ((rc = ptq8_engine_tensor_info(e, 0, i, shp)) != 0) return rc;
            buf.resize((size_t)n * shp[1] * shp[2] * shp[3]);
            if ((rc = ptq8_engine_dump(e, 0, i, n, buf.data(), buf.size())) != 0) return rc;
            dump(user, i, buf.data(), n, shp[1], shp[2], shp[3]);
        }
        return PTQ8_OK;
    } catch (const std::exception& ex) {
        return e->fail(std::string("forward_debug: ") + ex.what());
    }
}

int ptq8_capture_graph(ptq8_engine* e, int n) {
    if (!e) return PTQ8_ERR_INVALID;
    cudaGraphExec_t ge;
    return graph_for(e, n, &ge);
}

void ptq8_destroy(ptq8_engine* e) {
    if (!e) return;
    ptq8_model* m = e->owned_model;
    ptq8_engine_destroy(e);
    ptq8_model_free(m);   // after the engine, which points into it
}

const char* ptq8_last_error(const ptq8_engine* e) { return ptq8_engine_last_error(e); }

}  // extern "C"
