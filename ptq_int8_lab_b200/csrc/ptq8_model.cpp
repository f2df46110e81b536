// Strict loaders and topology validation for PTQW / PTQ2 / PTQC (see ptq8_model.hpp).
#include "ptq8_model.hpp"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sys/stat.h>
#include <iterator>
#include <limits>
#include <string>

namespace ptq8 {

namespace {

std::string fmt(const char* f, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, f);
    std::vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return std::string(buf);
}

bool fail(std::string* err, const std::string& m) {
    if (err) *err = m;
    return false;
}

constexpr uint64_t kMaxFileBytes = 1ull << 32;

// Bounds-checked little-endian reader over a whole file held in memory.
class Reader {
public:
    bool open(const std::string& path, std::string* err) {
        struct stat st {};
        if (::stat(path.c_str(), &st) != 0) return fail(err, "cannot open file: " + path);
        if (!S_ISREG(st.st_mode)) return fail(err, "not a regular file: " + path);
        if (st.st_size > (off_t)kMaxFileBytes) return fail(err, "file larger than 4 GiB: " + path);
        std::ifstream f(path, std::ios::binary);
        if (!f.is_open()) return fail(err, "cannot open file: " + path);
        f.seekg(0, std::ios::end);
        std::streamoff end = f.tellg();
        if (!f || end < 0 || end > (std::streamoff)kMaxFileBytes) return fail(err, "cannot read file size: " + path);
        buf_.resize((size_t)end);
        f.seekg(0, std::ios::beg);
        if (end > 0) f.read(reinterpret_cast<char*>(buf_.data()), end);
        if (!f) return fail(err, "read failed: " + path);
        return true;
    }
    size_t size() const { return buf_.size(); }
    size_t pos() const { return pos_; }
    size_t left() const { return buf_.size() - pos_; }
    bool raw(void* dst, size_t n, const char* what, std::string* err) {
        if (n > left())
            return fail(err, fmt("%s: file too short (needs %zu B, %zu B left of %zu) - truncated",
                                 what, n, left(), buf_.size()));
        std::memcpy(dst, buf_.data() + pos_, n);
        pos_ += n;
        return true;
    }
    bool i32(int* v, const char* what, std::string* err) {
        int32_t x;
        if (!raw(&x, 4, what, err)) return false;
        *v = x;
        return true;
    }
    bool floats(size_t n, std::vector<float>* v, const char* what, std::string* err) {
        if (n > left() / 4)
            return fail(err, fmt("%s: needs %zu floats (%zu B) but only %zu B left - truncated",
                                 what, n, n * 4, left()));
        v->resize(n);
        return raw(v->data(), n * 4, what, err);
    }

private:
    std::vector<uint8_t> buf_;
    size_t pos_ = 0;
};

bool mul_ok(size_t a, size_t b, size_t* out) {
    if (b != 0 && a > std::numeric_limits<size_t>::max() / b) return false;
    *out = a * b;
    return true;
}

bool conv_meta_ok(const ConvSpec& c, int i, std::string* err) {
    if (c.cout <= 0 || c.cin <= 0 || c.kh <= 0 || c.kw <= 0)
        return fail(err, fmt("conv[%d]: cout/cin/kh/kw must be positive (got %d/%d/%d/%d)",
                             i, c.cout, c.cin, c.kh, c.kw));
    if (c.sh < 1 || c.sw < 1 || c.ph < 0 || c.pw < 0)
        return fail(err, fmt("conv[%d]: stride must be >= 1 and padding >= 0 (%d,%d,%d,%d)",
                             i, c.sh, c.sw, c.ph, c.pw));
    if (c.relu != 0 && c.relu != 1 && c.relu != 2)
        return fail(err, fmt("conv[%d]: relu=%d invalid (0/1/2 only)", i, c.relu));
    if (c.groups < 1 || c.cout % c.groups != 0)
        return fail(err, fmt("conv[%d]: groups=%d invalid (needs groups >= 1 dividing cout=%d)",
                             i, c.groups, c.cout));
    return true;
}

bool read_conv_payload(Reader& r, ConvSpec& c, int i, std::string* err) {
    size_t nw = 0, t = 0;
    if (!mul_ok((size_t)c.cout, (size_t)c.cin, &t) || !mul_ok(t, (size_t)c.kh, &t) ||
        !mul_ok(t, (size_t)c.kw, &nw))
        return fail(err, fmt("conv[%d]: weight element count overflows", i));
    char what[64];
    std::snprintf(what, sizeof what, "conv[%d].weight", i);
    if (!r.floats(nw, &c.weight, what, err)) return false;
    std::snprintf(what, sizeof what, "conv[%d].bias", i);
    return r.floats((size_t)c.cout, &c.bias, what, err);
}

bool read_fc(Reader& r, Model& m, std::string* err) {
    if (!r.i32(&m.fc_in, "fc.fc_in", err) || !r.i32(&m.fc_out, "fc.fc_out", err)) return false;
    if (m.fc_in <= 0 || m.fc_out <= 0)
        return fail(err, fmt("fc_in/fc_out must be positive (got %d/%d)", m.fc_in, m.fc_out));
    size_t n = 0;
    if (!mul_ok((size_t)m.fc_in, (size_t)m.fc_out, &n)) return fail(err, "fc: element count overflows");
    if (!r.floats(n, &m.fc_w, "fc.weight", err)) return false;
    return r.floats((size_t)m.fc_out, &m.fc_b, "fc.bias", err);
}

bool load_ptqw(Reader& r, Model& m, std::string* err) {
    int n_conv = 0, n_block = 0;
    if (!r.i32(&n_conv, "header.n_conv", err) || !r.i32(&n_block, "header.n_block", err) ||
        !r.i32(&m.stem_pool, "header.stem_pool", err))
        return false;
    if (n_conv <= 0) return fail(err, "PTQW: n_conv must be > 0");
    if (n_block < 0) return fail(err, "PTQW: n_block is negative");
    if (m.stem_pool != 0 && m.stem_pool != 1) return fail(err, "PTQW: stem_pool must be 0/1");
    if ((size_t)n_conv * 36 > r.left()) return fail(err, "PTQW: n_conv exceeds the file size");
    m.convs.resize((size_t)n_conv);
    for (int i = 0; i < n_conv; i++) {
        ConvSpec& c = m.convs[i];
        int* meta[9] = {&c.cout, &c.cin, &c.kh, &c.kw, &c.sh, &c.sw, &c.ph, &c.pw, &c.relu};
        for (int k = 0; k < 9; k++) {
            char what[64];
            std::snprintf(what, sizeof what, "conv[%d].meta[%d]", i, k);
            if (!r.i32(meta[k], what, err)) return false;
        }
        c.groups = 1;
        if (!conv_meta_ok(c, i, err) || !read_conv_payload(r, c, i, err)) return false;
    }
    if ((size_t)n_block * 16 > r.left()) return fail(err, "PTQW: n_block exceeds the file size");
    m.blocks.resize((size_t)n_block);
    for (int i = 0; i < n_block; i++) {
        int c1, c2, ds, stride;
        if (!r.i32(&c1, "block.c1", err) || !r.i32(&c2, "block.c2", err) ||
            !r.i32(&ds, "block.ds", err) || !r.i32(&stride, "block.stride", err))
            return false;
        if (c1 < 0 || c1 >= n_conv || c2 < 0 || c2 >= n_conv)
            return fail(err, fmt("PTQW block[%d]: conv index out of range", i));
        if (ds < -1 || ds >= n_conv) return fail(err, fmt("PTQW block[%d]: ds=%d out of range", i, ds));
        if (stride < 1) return fail(err, fmt("PTQW block[%d]: stride < 1", i));
        BlockSpec& b = m.blocks[i];
        b.convs = {c1, c2};
        b.ds = ds;
        b.stride = stride;
        b.residual = 1;   // PTQW is the ResNet-18 block format: residual + ReLU
    }
    return read_fc(r, m, err);
}

// PTQ8 conv payload after the 10 meta ints: bits, f32 scales, f32 bias, codes (one byte
// each for W8, two per byte for W4), unpacked here to one code per byte.
bool read_native_payload(Reader& r, ConvSpec& c, int i, std::string* err) {
    char what[64];
    std::snprintf(what, sizeof what, "conv[%d].bits", i);
    if (!r.i32(&c.qbits, what, err)) return false;
    if (c.qbits != 8 && c.qbits != 4) return fail(err, fmt("conv[%d]: bits=%d (PTQ8 holds 8 or 4)", i, c.qbits));
    std::snprintf(what, sizeof what, "conv[%d].w_scale", i);
    if (!r.floats((size_t)c.cout, &c.wscale, what, err)) return false;
    for (int o = 0; o < c.cout; ++o)
        if (!std::isfinite(c.wscale[o]) || !(c.wscale[o] > 0.0f))
            return fail(err, fmt("conv[%d]: w_scale[%d] is not finite and positive", i, o));
    std::snprintf(what, sizeof what, "conv[%d].bias", i);
    if (!r.floats((size_t)c.cout, &c.bias, what, err)) return false;
    size_t k = 0, n = 0;
    if (!mul_ok((size_t)c.cin, (size_t)c.kh, &k) || !mul_ok(k, (size_t)c.kw, &k) || !mul_ok(k, (size_t)c.cout, &n))
        return fail(err, fmt("conv[%d]: code count overflows", i));
    const size_t row = c.qbits == 8 ? k : (k + 1) / 2;
    std::vector<uint8_t> raw;
    size_t nb = 0;
    if (!mul_ok(row, (size_t)c.cout, &nb)) return fail(err, fmt("conv[%d]: code bytes overflow", i));
    if (nb > r.left())
        return fail(err, fmt("conv[%d].codes: needs %zu B but only %zu B left - truncated", i, nb, r.left()));
    raw.resize(nb);
    std::snprintf(what, sizeof what, "conv[%d].codes", i);
    if (!r.raw(raw.data(), nb, what, err)) return false;
    c.codes.resize(n);
    for (int o = 0; o < c.cout; ++o)
        for (size_t j = 0; j < k; ++j) {
            int8_t v;
            if (c.qbits == 8) {
                v = (int8_t)raw[(size_t)o * row + j];
            } else {
                const int nib = (raw[(size_t)o * row + j / 2] >> (4 * (j & 1))) & 0xF;
                v = (int8_t)(nib >= 8 ? nib - 16 : nib);
            }
            c.codes[(size_t)o * k + j] = v;
        }
    return true;
}

// PTQ2 (and, with native = true, the PTQ8 package that shares its header, blocks and fc).
bool load_ptq2(Reader& r, Model& m, std::string* err, bool native = false) {
    if (r.size() < (native ? 24u : 20u)) return fail(err, "file too short: less than magic + header");
    if (native) {
        int version = 0;
        if (!r.i32(&version, "header.version", err)) return false;
        if (version != 1) return fail(err, fmt("PTQ8 version %d unsupported (1 only)", version));
    }
    int n_conv = 0, n_block = 0, ncp = 0;
    if (!r.i32(&n_conv, "header.n_conv", err) || !r.i32(&n_block, "header.n_block", err) ||
        !r.i32(&m.stem_pool, "header.stem_pool", err) || !r.i32(&ncp, "header.n_conv_per_block", err))
        return false;
    if (n_conv < 0) return fail(err, "header: n_conv is negative");
    if (n_conv == 0) return fail(err, "header: model has no conv");
    if (n_block < 0) return fail(err, "header: n_block is negative");
    if (m.stem_pool != 0 && m.stem_pool != 1) return fail(err, "header: stem_pool must be 0/1");
    if (ncp <= 0) return fail(err, "header: n_conv_per_block must be > 0");
    if ((size_t)n_block * (size_t)(ncp + 3) * 4 > r.size())
        return fail(err, "header: n_block x (ncp+3) exceeds the file size");
    if ((size_t)n_conv * 40 > r.left()) return fail(err, "header: n_conv exceeds the file size");
    m.convs.resize((size_t)n_conv);
    for (int i = 0; i < n_conv; i++) {
        ConvSpec& c = m.convs[i];
        int* meta[10] = {&c.cout, &c.cin, &c.kh, &c.kw, &c.sh, &c.sw, &c.ph, &c.pw, &c.relu, &c.groups};
        for (int k = 0; k < 10; k++) {
            char what[64];
            std::snprintf(what, sizeof what, "conv[%d].meta[%d]", i, k);
            if (!r.i32(meta[k], what, err)) return false;
        }
        if (!conv_meta_ok(c, i, err)) return false;
        if (!(native ? read_native_payload(r, c, i, err) : read_conv_payload(r, c, i, err))) return false;
    }
    m.blocks.resize((size_t)n_block);
    for (int i = 0; i < n_block; i++) {
        BlockSpec& b = m.blocks[i];
        std::vector<int> cs((size_t)ncp);
        for (int k = 0; k < ncp; k++) {
            char what[64];
            std::snprintf(what, sizeof what, "block[%d].conv[%d]", i, k);
            if (!r.i32(&cs[k], what, err)) return false;
            if (cs[k] < -1 || cs[k] >= n_conv)
                return fail(err, fmt("block[%d].conv[%d]=%d out of range (-1 padding or [0,%d))",
                                     i, k, cs[k], n_conv));
        }
        b.convs = cs;
        if (!r.i32(&b.ds, "block.ds", err)) return false;
        if (b.ds < -1 || b.ds >= n_conv)
            return fail(err, fmt("block[%d].ds=%d out of range (-1 or [0,%d))", i, b.ds, n_conv));
        if (!r.i32(&b.stride, "block.stride", err)) return false;
        if (b.stride < 1) return fail(err, fmt("block[%d].stride=%d < 1", i, b.stride));
        if (!r.i32(&b.residual, "block.residual", err)) return false;
        if (b.residual < 0 || b.residual > 2)
            return fail(err, fmt("block[%d].residual=%d invalid (0/1/2 only)", i, b.residual));
    }
    return read_fc(r, m, err);
}

}  // namespace

int conv_out_dim(int in, int k, int s, int p) { return (in + 2 * p - k) / s + 1; }

bool Model::load(const std::string& path, std::string* err) {
    Reader r;
    if (!r.open(path, err)) return false;
    char mg[4] = {0};
    if (r.size() < 4) return fail(err, path + ": shorter than 4 B, no magic");
    r.raw(mg, 4, "magic", err);
    Model m;
    bool ok;
    if (std::memcmp(mg, "PTQW", 4) == 0) {
        m.magic = "PTQW";
        ok = load_ptqw(r, m, err);
    } else if (std::memcmp(mg, "PTQ2", 4) == 0) {
        m.magic = "PTQ2";
        ok = load_ptq2(r, m, err);
    } else if (std::memcmp(mg, "PTQ8", 4) == 0) {
        m.magic = "PTQ8";
        ok = load_ptq2(r, m, err, true);
    } else {
        std::string p;
        for (int i = 0; i < 4; i++) {
            unsigned char ch = (unsigned char)mg[i];
            if (ch >= 32 && ch < 127) p.push_back((char)ch);
            else p += fmt("\\x%02x", ch);
        }
        return fail(err, path + ": bad magic (expected PTQW/PTQ2/PTQ8, got '" + p + "')");
    }
    if (!ok) return false;
    if (r.pos() != r.size())
        return fail(err, fmt("%s EOF check failed: parse ended at %zu B of %zu B - %zu trailing bytes rejected",
                             m.magic.c_str(), r.pos(), r.size(), r.size() - r.pos()));
    if (!m.validate(err)) return false;
    *this = std::move(m);
    if (err) err->clear();
    return true;
}

bool Model::validate(std::string* err, int input_h, int input_w) const {
    if (convs.empty()) return fail(err, "model has no conv");
    if (fc_in <= 0 || fc_out <= 0) return fail(err, "fc_in/fc_out must be positive");
    const ConvSpec& stem = convs[0];
    int ch = stem.cout;
    int hh = conv_out_dim(input_h, stem.kh, stem.sh, stem.ph);
    int ww = conv_out_dim(input_w, stem.kw, stem.sw, stem.pw);
    if (hh <= 0 || ww <= 0) return fail(err, "stem output is empty");
    if (stem_pool) {
        hh = (hh + 2 - 3) / 2 + 1;
        ww = (ww + 2 - 3) / 2 + 1;
    }
    for (size_t bi = 0; bi < blocks.size(); bi++) {
        const BlockSpec& b = blocks[bi];
        bool saw_pad = false, any = false;
        int tch = ch, th = hh, tw = ww;
        for (size_t k = 0; k < b.convs.size(); k++) {
            int ci = b.convs[k];
            if (ci == -1) { saw_pad = true; continue; }
            if (saw_pad)
                return fail(err, fmt("block[%zu]: -1 padding must be at the tail (conv at %zu after padding)", bi, k));
            if (ci < 0 || ci >= (int)convs.size())
                return fail(err, fmt("block[%zu]: conv index %d out of range", bi, ci));
            const ConvSpec& c = convs[ci];
            if (c.in_channels() != tch)
                return fail(err, fmt("block[%zu] conv[%zu] input channels %d != upstream %d (cin=%d, groups=%d)",
                                     bi, k, c.in_channels(), tch, c.cin, c.groups));
            th = conv_out_dim(th, c.kh, c.sh, c.ph);
            tw = conv_out_dim(tw, c.kw, c.sw, c.pw);
            if (th <= 0 || tw <= 0) return fail(err, fmt("block[%zu]: empty output map", bi));
            tch = c.cout;
            any = true;
        }
        if (!any) return fail(err, fmt("block[%zu] has no valid conv", bi));
        if (b.residual == 0) {
            if (b.ds >= 0) return fail(err, fmt("block[%zu]: residual=0 but a ds conv is given", bi));
        } else {
            int ich = ch, ih = hh, iw = ww;
            if (b.ds >= 0) {
                const ConvSpec& d = convs[b.ds];
                if (d.in_channels() != ch)
                    return fail(err, fmt("block[%zu] ds input channels %d != upstream %d", bi, d.in_channels(), ch));
                ih = conv_out_dim(ih, d.kh, d.sh, d.ph);
                iw = conv_out_dim(iw, d.kw, d.sw, d.pw);
                ich = d.cout;
            }
            if (tch != ich || th != ih || tw != iw)
                return fail(err, fmt("block[%zu]: residual shape mismatch: main (%d,%d,%d) vs identity (%d,%d,%d)",
                                     bi, tch, th, tw, ich, ih, iw));
        }
        ch = tch; hh = th; ww = tw;
    }
    if (ch != fc_in) return fail(err, fmt("fc_in=%d != topology output channels %d", fc_in, ch));
    if ((size_t)fc_in * (size_t)fc_out != fc_w.size()) return fail(err, "fc weight count mismatch");
    if ((size_t)fc_out != fc_b.size()) return fail(err, "fc bias count mismatch");
    return true;
}

bool load_ptqc(const std::string& path, size_t n_expected,
               std::vector<std::pair<float, float>>* out, std::string* err) {
    Reader r;
    if (!r.open(path, err)) return false;
    if (r.size() < 8) return fail(err, fmt("PTQC file too short: %zu B (needs at least 8 B magic+n)", r.size()));
    char mg[4];
    int n = -1;
    r.raw(mg, 4, "magic", err);
    r.i32(&n, "n", err);
    if (std::memcmp(mg, "PTQC", 4) != 0) return fail(err, "PTQC magic mismatch (expected \"PTQC\")");
    if (n < 0) return fail(err, fmt("PTQC n=%d is negative", n));
    size_t want = 8 + 8 * (size_t)n;
    if (r.size() != want)
        return fail(err, fmt("PTQC length mismatch: file %zu B, n=%d needs %zu B (8+8n; truncation or trailing bytes rejected)",
                             r.size(), n, want));
    if ((size_t)n != n_expected)
        return fail(err, fmt("PTQC layer count mismatch: n=%d != model conv count %zu", n, n_expected));
    out->resize((size_t)n);
    for (int i = 0; i < n; i++) {
        float lo, hi;
        r.raw(&lo, 4, "lo", err);
        r.raw(&hi, 4, "hi", err);
        if (!std::isfinite(lo) || !std::isfinite(hi))
            return fail(err, fmt("PTQC layer %d range not finite: lo=%g hi=%g", i, lo, hi));
        if (lo > hi) return fail(err, fmt("PTQC layer %d range invalid: lo=%g > hi=%g", i, lo, hi));
        (*out)[i] = {lo, hi};
    }
    if (err) err->clear();
    return true;
}

double act_scale_from_range(float lo, float hi, int bits, int mode) {
    const int qmax = (1 << (bits - 1)) - 1;
    double s;
    if (mode == ACT_MINMAX) s = ((double)hi - (double)lo) / qmax;
    else s = std::fmax(std::fabs((double)lo), std::fabs((double)hi)) / qmax;
    return s < 1e-8 ? 1e-8 : s;
}

static inline double round_half_away(double v) { return v >= 0.0 ? std::floor(v + 0.5) : std::ceil(v - 0.5); }

void quantize_weight_per_channel(const float* w, int cout, int k, int bits, int8_t* codes, float* scale32) {
    const int qmax = (1 << (bits - 1)) - 1;
    const double qmin = -(double)(qmax + 1);
    for (int o = 0; o < cout; o++) {
        const float* row = w + (size_t)o * k;
        double amax = 0.0;
        for (int i = 0; i < k; i++) amax = std::fmax(amax, std::fabs((double)row[i]));
        double s = amax / qmax;
        if (s < 1e-8) s = 1e-8;
        scale32[o] = (float)s;
        for (int i = 0; i < k; i++) {
            double v = round_half_away((double)row[i] / s);
            if (v < qmin) v = qmin;
            if (v > qmax) v = qmax;
            codes[(size_t)o * k + i] = (int8_t)v;
        }
    }
}


// ---------------------------------------------------------------- layer plan JSON

namespace {

// A small strict JSON reader (RFC 8259 values; strings without \u escapes
// beyond the ASCII range), enough for the layer-plan files.
struct JValue {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<JValue> arr;
    std::vector<std::pair<std::string, JValue>> obj;
    const JValue* get(const char* key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const std::string& t;
    size_t i = 0;
    std::string err;
    explicit JParser(const std::string& text) : t(text) {}
    void ws() {
        while (i < t.size() && (t[i] == ' ' || t[i] == '\n' || t[i] == '\r' || t[i] == '\t')) ++i;
    }
    bool fail(const char* what) {
        if (err.empty()) err = fmt("JSON: %s at byte %zu", what, i);
        return false;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (t.compare(i, n, w) != 0) return fail("bad literal");
        i += n;
        return true;
    }
    bool string(std::string* out) {
        if (t[i] != '"') return fail("expected string");
        ++i;
        out->clear();
        while (i < t.size() && t[i] != '"') {
            char c = t[i++];
            if (c == '\\') {
                if (i >= t.size()) return fail("bad escape");
                const char e = t[i++];
                switch (e) {
                    case '"': case '\\': case '/': c = e; break;
                    case 'b': c = '\b'; break;
                    case 'f': c = '\f'; break;
                    case 'n': c = '\n'; break;
                    case 'r': c = '\r'; break;
                    case 't': c = '\t'; break;
                    case 'u': {
                        if (i + 4 > t.size()) return fail("bad \\u escape");
                        const unsigned v = static_cast<unsigned>(std::strtoul(t.substr(i, 4).c_str(), nullptr, 16));
                        i += 4;
                        if (v > 0x7f) return fail("non-ASCII \\u escape");
                        c = static_cast<char>(v);
                        break;
                    }
                    default: return fail("bad escape");
                }
            }
            out->push_back(c);
        }
        if (i >= t.size()) return fail("unterminated string");
        ++i;
        return true;
    }
    bool value(JValue* v, int depth) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (i >= t.size()) return fail("unexpected end");
        const char c = t[i];
        if (c == '{') {
            v->kind = JValue::OBJ;
            ++i;
            ws();
            if (i < t.size() && t[i] == '}') { ++i; return true; }
            while (true) {
                ws();
                std::string key;
                if (i >= t.size() || !string(&key)) return fail("expected key");
                ws();
                if (i >= t.size() || t[i] != ':') return fail("expected ':'");
                ++i;
                v->obj.emplace_back(key, JValue());
                if (!value(&v->obj.back().second, depth + 1)) return false;
                ws();
                if (i < t.size() && t[i] == ',') { ++i; continue; }
                if (i < t.size() && t[i] == '}') { ++i; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v->kind = JValue::ARR;
            ++i;
            ws();
            if (i < t.size() && t[i] == ']') { ++i; return true; }
            while (true) {
                v->arr.emplace_back();
                if (!value(&v->arr.back(), depth + 1)) return false;
                ws();
                if (i < t.size() && t[i] == ',') { ++i; continue; }
                if (i < t.size() && t[i] == ']') { ++i; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v->kind = JValue::STR;
            return string(&v->str);
        }
        if (c == 't') { v->kind = JValue::BOOL; v->b = true; return lit("true"); }
        if (c == 'f') { v->kind = JValue::BOOL; v->b = false; return lit("false"); }
        if (c == 'n') { v->kind = JValue::NUL; return lit("null"); }
        if (c == '-' || (c >= '0' && c <= '9')) {
            const char* s0 = t.c_str() + i;
            char* end = nullptr;
            v->kind = JValue::NUM;
            v->num = std::strtod(s0, &end);
            if (end == s0) return fail("bad number");
            i += static_cast<size_t>(end - s0);
            return true;
        }
        return fail("unexpected character");
    }
};

}  // namespace

bool load_layer_plan(const std::string& path, size_t n_conv, std::vector<int>* bits, std::string* err) {
    struct stat st {};
    if (::stat(path.c_str(), &st) != 0 || !S_ISREG(st.st_mode) || st.st_size > (off_t)(64u << 20)) {
        *err = "cannot open layer plan (not a regular file of at most 64 MiB): " + path;
        return false;
    }
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        *err = "cannot open " + path;
        return false;
    }
    std::string text((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    JParser p(text);
    JValue doc;
    if (!p.value(&doc, 0)) {
        *err = path + ": " + p.err;
        return false;
    }
    p.ws();
    if (p.i != text.size()) {
        *err = path + ": trailing data after the JSON document";
        return false;
    }
    const JValue* layers = doc.kind == JValue::OBJ ? doc.get("layers") : nullptr;
    if (!layers || layers->kind != JValue::ARR || layers->arr.size() != n_conv) {
        *err = fmt("%s: 'layers' must list %zu convs in engine order", path.c_str(), n_conv);
        return false;
    }
    bits->clear();
    for (size_t k = 0; k < n_conv; ++k) {
        const JValue& e = layers->arr[k];
        const JValue* b = e.kind == JValue::OBJ ? e.get("bits") : nullptr;
        const int v = b && b->kind == JValue::NUM ? static_cast<int>(b->num) : 0;
        if (v != 4 && v != 8) {
            *err = fmt("%s: layer %zu bits=%d (only 4 / 8)", path.c_str(), k, v);
            return false;
        }
        const JValue* sc = e.get("scheme");
        if (sc && (sc->kind != JValue::STR || sc->str != "per_channel")) {
            *err = fmt("%s: layer %zu scheme %s: only per_channel weights run on the engine", path.c_str(), k,
                        sc->kind == JValue::STR ? sc->str.c_str() : "(not a string)");
            return false;
        }
        bits->push_back(v);
    }
    return true;
}

}  // namespace ptq8
