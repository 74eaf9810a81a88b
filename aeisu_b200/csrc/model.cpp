// Checkpoint loaders.  The folded layout follows aeisu/model.py:554-583; the SPYR8
// container follows the reference loader optimized/native/src/neural/srcpyr/SrcPyrModel.cpp
// (header 37-68, descriptors 70-80, checks 243-470), restated for Linux with a portable
// SHA-256 in place of BCrypt.
#include "model.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <tuple>

#include "common.h"
#include "sha256.h"

namespace aeisu {

const LayerSpec kLayerSpecs[kLayerCount] = {
    {32, 32, 1, 1, "project"},      {64, 128, 1, 1, "compress"},    {64, 32, 3, 2, "bottleneck0"},
    {64, 32, 3, 2, "bottleneck1"},  {64, 32, 3, 2, "bottleneck2"},  {64, 32, 3, 2, "bottleneck3"},
    {128, 64, 1, 1, "expand"},      {64, 32, 3, 1, "refine"},       {64, 64, 1, 1, "tail"},
};

static size_t weight_count(const LayerSpec& s) { return size_t(s.cout) * s.cin_per_group * s.k * s.k; }

uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return uint16_t(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
    if (ax >= 0x477ff000u) return uint16_t(sign | 0x7c00u);  // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {                                    // half subnormal or zero
        if (ax < 0x33000000u) return uint16_t(sign);           // < 2^-25: rounds to 0
        const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
        const int shift = 126 - int(ax >> 23);                 // 14 .. 24
        uint32_t q = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return uint16_t(sign | q);
    }
    uint32_t h = ((ax >> 13) - (112u << 10));
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return uint16_t(sign | h);
}

float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {
            float v = std::ldexp(float(m), -24);
            std::memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

float e4m3_to_f32(uint8_t c) {
    const float sign = (c & 0x80) ? -1.f : 1.f;
    const int e = (c >> 3) & 0xf, m = c & 7;
    if (e == 15 && m == 7) return std::nanf("");
    if (e == 0) return sign * std::ldexp(float(m), -9);
    return sign * std::ldexp(1.f + m / 8.f, e - 7);
}

// ---- folded .pt layout --------------------------------------------------------------

HostModel load_folded(const float* v, size_t count, float l1_scale) {
    require(v != nullptr, "folded weights pointer is null");
    require(count == AEISU_FOLDED_VALUES,
            "folded checkpoint must hold " + std::to_string(AEISU_FOLDED_VALUES) + " values, got " +
                std::to_string(count));
    require(std::isfinite(l1_scale) && l1_scale > 0, "basis_l1_scale must be positive and finite");
    for (size_t i = 0; i < count; ++i)
        require(std::isfinite(v[i]), "folded checkpoint holds a non-finite value", AEISU_ERR_BAD_ARTIFACT);
    HostModel m;
    m.format = "folded";
    m.architecture = "aeisu_parallel32x4_folded_v1";
    size_t o = 0;
    auto take = [&](float* dst, size_t n) { std::memcpy(dst, v + o, n * 4); o += n; };
    take(m.stencil, 9);        // analysis_rgb_basis
    take(m.stencil + 9, 3);    // analysis_rgb_mix
    take(m.stencil + 12, 3);   // analysis_dx_rows
    take(m.stencil + 15, 3);   // analysis_dy_cols
    take(m.stencil + 18, 3);   // analysis_diag45
    take(m.stencil + 21, 3);   // analysis_diag135
    take(m.base, 100);         // base_kernel [25,4]
    std::vector<float> raw(16 * 4 * 25);
    take(raw.data(), raw.size());  // basis_raw [16,4,25]
    // project_basis (reconstruction.py:8-12): centre each 25-tap vector, scale to L1,
    // permute [k, phase, tap] -> [tap, k, phase].
    for (int k = 0; k < 16; ++k)
        for (int p = 0; p < 4; ++p) {
            const float* r = &raw[(k * 4 + p) * 25];
            float sum = 0.f;
            for (int t = 0; t < 25; ++t) sum += r[t];
            const float mean = sum / 25.f;
            float c[25], l1 = 0.f;
            for (int t = 0; t < 25; ++t) { c[t] = r[t] - mean; l1 += std::fabs(c[t]); }
            const float f = l1_scale / std::max(l1, 1e-6f);
            for (int t = 0; t < 25; ++t) m.basis[(t * 16 + k) * 4 + p] = c[t] * f;
        }
    // convolutions in CONVOLUTIONS order: project, compress, a1..a4, b1..b4, expand, refine, head
    auto read_conv = [&](size_t wn, size_t bn, std::vector<float>& w, std::vector<float>& b) {
        w.assign(v + o, v + o + wn); o += wn;
        b.assign(v + o, v + o + bn); o += bn;
    };
    std::vector<float> aw[4], ab[4], bw[4], bb[4];
    read_conv(32 * 32, 32, m.layers[kProject].w, m.layers[kProject].bias);
    read_conv(64 * 128, 64, m.layers[kCompress].w, m.layers[kCompress].bias);
    for (int i = 0; i < 4; ++i) read_conv(32 * 32 * 9, 32, aw[i], ab[i]);
    for (int i = 0; i < 4; ++i) read_conv(32 * 32 * 9, 32, bw[i], bb[i]);
    read_conv(128 * 64, 128, m.layers[kExpand].w, m.layers[kExpand].bias);
    read_conv(64 * 32 * 9, 64, m.layers[kRefine].w, m.layers[kRefine].bias);
    read_conv(64 * 64, 64, m.layers[kTail].w, m.layers[kTail].bias);
    if (o != count) fail(AEISU_ERR_BAD_ARTIFACT, "folded layout size mismatch");
    for (int i = 0; i < 4; ++i) {
        LayerWeights& L = m.layers[kCore0 + i];
        L.w = aw[i];
        L.w.insert(L.w.end(), bw[i].begin(), bw[i].end());
        L.bias = ab[i];
        L.bias.insert(L.bias.end(), bb[i].begin(), bb[i].end());
    }
    for (int l = 0; l < kLayerCount; ++l) {
        LayerWeights& L = m.layers[l];
        L.bias_fp8 = L.bias;
        L.slope.assign(kLayerSpecs[l].cout, l == kTail ? 1.0f : 0.1f);
        L.w_fp16.resize(L.w.size());
        for (size_t i = 0; i < L.w.size(); ++i) L.w_fp16[i] = f32_to_f16_bits(L.w[i]);
    }
    return m;
}

// ---- SPYR8 v1 ----------------------------------------------------------------------

namespace {

constexpr char kArchitecture[] = "aif16x5_learnedrgb4dir8_s32_parallel32x4_learnedbase_oc25_v1";
constexpr size_t kHeaderSize = 512, kDescriptorSize = 80, kChecksumOffset = 184, kAlign = 64;
enum : uint32_t { kFp8 = 1, kFp16 = 2, kFp32 = 3, kNvFp4 = 4, kNvFp4Block16 = 5 };
enum : uint32_t { kVector = 1, kOihw = 2, kAdaptiveBasis = 4 };

struct View {
    uint32_t dtype = 0, layout = 0, rank = 0, shape[4] = {0, 0, 0, 0};
    const uint8_t* data = nullptr;
    uint64_t bytes = 0;
};

template <typename T> T rd(const uint8_t* p) { T v; std::memcpy(&v, p, sizeof(T)); return v; }

std::string fixed_string(const uint8_t* p, size_t cap, const char* field) {
    const void* end = std::memchr(p, 0, cap);
    if (!end) fail(AEISU_ERR_BAD_ARTIFACT, std::string("unterminated SPYR8 ") + field);
    return std::string(reinterpret_cast<const char*>(p), static_cast<const uint8_t*>(end) - p);
}

std::string hex(const uint8_t* b, size_t n) {
    static const char* d = "0123456789abcdef";
    std::string s;
    for (size_t i = 0; i < n; ++i) { s += d[b[i] >> 4]; s += d[b[i] & 15]; }
    return s;
}

const View& need(const std::map<std::string, View>& t, const std::string& name, uint32_t dtype,
                 uint32_t layout, std::initializer_list<uint32_t> shape) {
    auto it = t.find(name);
    if (it == t.end()) fail(AEISU_ERR_BAD_ARTIFACT, "missing SPYR8 tensor: " + name);
    const View& v = it->second;
    if (v.dtype != dtype || v.layout != layout || v.rank != shape.size())
        fail(AEISU_ERR_BAD_ARTIFACT, "SPYR8 tensor metadata mismatch: " + name);
    size_t i = 0;
    for (uint32_t s : shape)
        if (v.shape[i++] != s) fail(AEISU_ERR_BAD_ARTIFACT, "SPYR8 tensor shape mismatch: " + name);
    return v;
}

std::vector<float> floats(const View& v) {
    std::vector<float> out(v.bytes / 4);
    std::memcpy(out.data(), v.data, v.bytes);
    for (float f : out)
        if (!std::isfinite(f)) fail(AEISU_ERR_BAD_ARTIFACT, "non-finite SPYR8 FP32 tensor value");
    return out;
}

}  // namespace

HostModel load_spyr8(const uint8_t* data, size_t size) {
    require(data != nullptr, "SPYR8 data pointer is null");
    if (size < kHeaderSize) fail(AEISU_ERR_BAD_ARTIFACT, "SPYR8 artifact is smaller than its header");
    const uint8_t* h = data;
    static const char magic[8] = {'S', 'P', 'Y', 'R', '8', 'F', '8', '\0'};
    if (std::memcmp(h, magic, 8) != 0 || rd<uint32_t>(h + 8) != 1 || rd<uint32_t>(h + 12) != kHeaderSize ||
        rd<uint32_t>(h + 16) != 0x01020304u || rd<uint32_t>(h + 20) != 0)
        fail(AEISU_ERR_BAD_ARTIFACT, "unsupported SPYR8 magic/version/endian/flags");
    const std::string arch = fixed_string(h + 24, 64, "architecture");
    if (arch != kArchitecture)
        fail(AEISU_ERR_UNSUPPORTED, "unsupported SPYR8 architecture: " + arch);
    const uint32_t count = rd<uint32_t>(h + 132);
    const uint64_t file_size = rd<uint64_t>(h + 152), toc = rd<uint64_t>(h + 160),
                   toc_bytes = rd<uint64_t>(h + 168), payload = rd<uint64_t>(h + 176);
    const uint32_t expect_u32[11] = {8, 32, 32, 64, 4, 64, 2, 1, 1, kOihw, 1};
    bool ok = true;
    for (int i = 0; i < 11; ++i) ok &= rd<uint32_t>(h + 88 + 4 * i) == expect_u32[i];
    ok &= count >= 59u && rd<uint32_t>(h + 136) == kAlign && rd<uint32_t>(h + 140) == kDescriptorSize;
    ok &= file_size == size && toc == kHeaderSize && toc_bytes == uint64_t(count) * kDescriptorSize;
    const uint64_t toc_end = (toc + toc_bytes + kAlign - 1) / kAlign * kAlign;
    ok &= payload >= toc_end && payload <= file_size;
    if (!ok) fail(AEISU_ERR_BAD_ARTIFACT, "unsupported or inconsistent SPYR8 header");
    for (size_t i = 216; i < kHeaderSize; ++i)
        if (h[i]) fail(AEISU_ERR_BAD_ARTIFACT, "nonzero SPYR8 v1 header extension bytes");
    Sha256 sha;
    sha.update(data, kChecksumOffset);
    const uint8_t zeros[32] = {};
    sha.update(zeros, 32);
    sha.update(data + kChecksumOffset + 32, size - kChecksumOffset - 32);
    const auto digest = sha.finish();
    if (std::memcmp(digest.data(), h + kChecksumOffset, 32) != 0)
        fail(AEISU_ERR_BAD_ARTIFACT, "SPYR8 artifact checksum mismatch: expected " +
                                         hex(h + kChecksumOffset, 32) + ", observed " + hex(digest.data(), 32));
    const float edge_shift = rd<float>(h + 144), edge_gain = rd<float>(h + 148);
    if (!std::isfinite(edge_shift) || edge_shift < 0 || !std::isfinite(edge_gain) || edge_gain < 0)
        fail(AEISU_ERR_BAD_ARTIFACT, "invalid SPYR8 edge-phase parameters");

    std::map<std::string, View> tensors;
    std::vector<std::tuple<uint64_t, uint64_t>> ranges;
    for (uint32_t i = 0; i < count; ++i) {
        const uint64_t off = toc + uint64_t(i) * kDescriptorSize;
        if (off + kDescriptorSize > size) fail(AEISU_ERR_BAD_ARTIFACT, "SPYR8 tensor descriptor out of bounds");
        const uint8_t* d = data + off;
        const std::string name = fixed_string(d, 32, "tensor name");
        View v;
        v.dtype = rd<uint32_t>(d + 32);
        v.layout = rd<uint32_t>(d + 36);
        v.rank = rd<uint32_t>(d + 40);
        if (name.empty() || tensors.count(name) || v.rank == 0 || v.rank > 4)
            fail(AEISU_ERR_BAD_ARTIFACT, "invalid or duplicate SPYR8 tensor descriptor");
        uint64_t elements = 1;
        for (int k = 0; k < 4; ++k) {
            v.shape[k] = rd<uint32_t>(d + 44 + 4 * k);
            if (uint32_t(k) < v.rank) {
                if (v.shape[k] == 0) fail(AEISU_ERR_BAD_ARTIFACT, "invalid SPYR8 tensor dimensions: " + name);
                elements *= v.shape[k];
            } else if (v.shape[k] != 0) {
                fail(AEISU_ERR_BAD_ARTIFACT, "nonzero unused SPYR8 dimension: " + name);
            }
        }
        uint64_t esize;
        switch (v.dtype) {
            case kFp8: case kNvFp4: esize = 1; break;
            case kFp16: case kNvFp4Block16: esize = 2; break;
            case kFp32: esize = 4; break;
            default: fail(AEISU_ERR_BAD_ARTIFACT, "unsupported SPYR8 tensor dtype: " + name);
        }
        const uint64_t expected = v.dtype == kNvFp4 ? (elements + 1) / 2 : elements * esize;
        const uint64_t toff = rd<uint64_t>(d + 60), tbytes = rd<uint64_t>(d + 68);
        const bool reserved_zero = !d[76] && !d[77] && !d[78] && !d[79];
        if (toff % kAlign || toff < payload || tbytes == 0 || toff > file_size ||
            tbytes > file_size - toff || tbytes != expected || !reserved_zero)
            fail(AEISU_ERR_BAD_ARTIFACT, "SPYR8 tensor bounds or byte count mismatch: " + name);
        v.data = data + toff;
        v.bytes = tbytes;
        tensors.emplace(name, v);
        ranges.emplace_back(toff, toff + tbytes);
    }
    std::sort(ranges.begin(), ranges.end());
    for (size_t i = 1; i < ranges.size(); ++i)
        if (std::get<1>(ranges[i - 1]) > std::get<0>(ranges[i]))
            fail(AEISU_ERR_BAD_ARTIFACT, "overlapping SPYR8 tensor payloads");

    HostModel m;
    m.format = "spyr8";
    m.architecture = arch;
    m.checksum_hex = hex(digest.data(), 32);
    m.has_fp8 = true;
    const auto scales = floats(need(tensors, "activation_scales", kFp32, kVector, {10}));
    std::copy(scales.begin(), scales.end(), m.act_scales);
    const auto basis = floats(need(tensors, "adaptive_basis", kFp32, kAdaptiveBasis, {25, 16, 4}));
    const auto base = floats(need(tensors, "adaptive_base", kFp32, kAdaptiveBasis, {25, 4}));
    const auto stencil = floats(need(tensors, "analysis_stencil", kFp32, kVector, {24}));
    const auto guards = floats(need(tensors, "precision_guards", kFp32, kVector, {2}));
    for (float g : guards)
        if (g != 0.f && g != 1.f) fail(AEISU_ERR_BAD_ARTIFACT, "Invalid adaptive precision policy");
    for (int kp = 0; kp < 64; ++kp) {
        float dc = 0.f, l1 = 0.f;
        for (int t = 0; t < 25; ++t) { dc += basis[t * 64 + kp]; l1 += std::fabs(basis[t * 64 + kp]); }
        if (std::fabs(dc) > 1e-5f || l1 > 0.5001f)
            fail(AEISU_ERR_BAD_ARTIFACT, "Adaptive basis violates zero-DC/L1 contract");
    }
    std::copy(basis.begin(), basis.end(), m.basis);
    std::copy(base.begin(), base.end(), m.base);
    std::copy(stencil.begin(), stencil.end(), m.stencil);
    for (int l = 0; l < kLayerCount; ++l) {
        const LayerSpec& s = kLayerSpecs[l];
        const std::string p = s.spyr_name;
        const uint32_t co = s.cout, ci = s.cin_per_group, k = s.k;
        const View& w8 = need(tensors, p + ".weight_fp8", kFp8, kOihw, {co, ci, k, k});
        const View& w16 = need(tensors, p + ".weight_fp16", kFp16, kOihw, {co, ci, k, k});
        LayerWeights& L = m.layers[l];
        L.w_scale = floats(need(tensors, p + ".weight_scale", kFp32, kVector, {co}));
        L.bias = floats(need(tensors, p + ".bias", kFp32, kVector, {co}));
        L.slope = floats(need(tensors, p + ".prelu", kFp32, kVector, {co}));
        L.bias_fp8 = floats(need(tensors, p + ".bias_fp8", kFp32, kVector, {co}));
        L.w_fp8.assign(w8.data, w8.data + w8.bytes);
        L.w_fp16.resize(weight_count(s));
        std::memcpy(L.w_fp16.data(), w16.data, w16.bytes);
        L.w.resize(L.w_fp16.size());
        for (size_t i = 0; i < L.w.size(); ++i) {
            L.w[i] = f16_bits_to_f32(L.w_fp16[i]);
            if (!std::isfinite(L.w[i])) fail(AEISU_ERR_BAD_ARTIFACT, "non-finite FP16 weight in " + p);
        }
        for (uint8_t c : L.w_fp8)
            if ((c & 0x7f) == 0x7f) fail(AEISU_ERR_BAD_ARTIFACT, "NaN FP8 weight in " + p);
    }
    return m;
}

HostModel load_int8(const aeisu_int8_artifact& a) {
    // Checks of MixedRuntime.__init__ (optimized/shader/runtime.py:37-59) that concern the
    // arrays themselves; the format and precision policy are checked by the caller, which
    // reads the .pt record.
    auto bad = [](const std::string& msg) { fail(AEISU_ERR_BAD_ARTIFACT, "INT8 artifact: " + msg); };
    auto finite = [&](const float* p, size_t n, const char* what) {
        if (!p) bad(std::string(what) + " is missing");
        for (size_t i = 0; i < n; ++i)
            if (!std::isfinite(p[i])) bad(std::string(what) + " has a non-finite value");
    };
    HostModel m;
    m.format = "shader_int8";
    m.architecture = "shader_precision_v1 int8/fp16";
    m.has_int8 = true;
    finite(a.analysis, 24, "analysis_parameters");
    finite(a.base, 100, "base");
    finite(a.bank, 1600, "bank");
    finite(a.activation_scales, 10, "activation_scales");
    std::copy(a.analysis, a.analysis + 24, m.stencil);
    std::copy(a.base, a.base + 100, m.base);
    std::copy(a.bank, a.bank + 1600, m.basis);
    for (int i = 0; i < 10; ++i) {
        if (!(a.activation_scales[i] > 0.f)) bad("activation scales must be positive");
        m.act_scales[i] = a.activation_scales[i];
    }
    auto half_layer = [&](int l, const uint16_t* w, const float* b, const char* name) {
        const LayerSpec& sp = kLayerSpecs[l];
        const size_t n = size_t(sp.cout) * sp.cin_per_group * sp.k * sp.k;
        if (!w) bad(std::string(name) + " weights are missing");
        LayerWeights& L = m.layers[l];
        L.w_fp16.assign(w, w + n);
        L.w.resize(n);
        for (size_t i = 0; i < n; ++i) {
            L.w[i] = f16_bits_to_f32(w[i]);
            if (!std::isfinite(L.w[i])) bad(std::string(name) + " weights have a non-finite value");
        }
        finite(b, sp.cout, name);
        L.bias.assign(b, b + sp.cout);
        L.bias_fp8 = L.bias;
        L.slope.assign(sp.cout, l == kTail ? 1.0f : 0.1f);
    };
    half_layer(kProject, a.project_w, a.project_b, "project");
    half_layer(kRefine, a.refine_w, a.refine_b, "refine");
    half_layer(kTail, a.tail_w, a.tail_b, "tail");
    static const int kInt8Layers[6] = {kCompress, kCore0, kCore1, kCore2, kCore3, kExpand};
    static const char* kNames[6] = {"compress", "bottleneck0", "bottleneck1", "bottleneck2", "bottleneck3", "expand"};
    for (int i = 0; i < 6; ++i) {
        const int l = kInt8Layers[i];
        const LayerSpec& sp = kLayerSpecs[l];
        const size_t n = size_t(sp.cout) * sp.cin_per_group * sp.k * sp.k;
        if (!a.int8_w[i]) bad(std::string(kNames[i]) + " weights are missing");
        finite(a.int8_factor[i], sp.cout, kNames[i]);
        finite(a.int8_bias[i], sp.cout, kNames[i]);
        LayerWeights& L = m.layers[l];
        L.w.resize(n);
        L.w_fp16.resize(n);
        for (size_t k = 0; k < n; ++k) {
            const int q = a.int8_w[i][k];
            if (q < -127 || q > 127) bad(std::string(kNames[i]) + " has a weight code outside [-127, 127]");
            L.w[k] = float(q);
            L.w_fp16[k] = f32_to_f16_bits(float(q));   // exact: |q| <= 127
        }
        L.factor.assign(a.int8_factor[i], a.int8_factor[i] + sp.cout);
        L.bias.assign(a.int8_bias[i], a.int8_bias[i] + sp.cout);
        L.bias_fp8 = L.bias;
        L.slope.assign(sp.cout, 0.1f);
    }
    return m;
}

}  // namespace aeisu
