#include "tc_pack.h"

#include "common.h"

namespace aeisu {
namespace {

size_t append_bytes(std::vector<uint8_t>& dst, const std::vector<uint8_t>& img) {
    while (dst.size() % 128) dst.push_back(0);
    const size_t at = dst.size();
    dst.insert(dst.end(), img.begin(), img.end());
    return at;
}

size_t append_floats(std::vector<float>& dst, const std::vector<float>& v) {
    while (dst.size() % 32) dst.push_back(0.f);
    const size_t at = dst.size();
    dst.insert(dst.end(), v.begin(), v.end());
    return at;
}

float round_f16(float v) { return f16_bits_to_f32(f32_to_f16_bits(v)); }

}  // namespace

TcHostPack pack_tc(const HostModel& m, int route) {
    const bool fp8 = route == kRouteE4M3, i8 = route == kRouteI8;
    require(!fp8 || m.has_fp8, "the mixed route needs the FP8 weights and scales of a SPYR8 artifact",
            AEISU_ERR_UNSUPPORTED);
    require(i8 == m.has_int8, "the INT8 route needs, and only runs, the INT8 artifact", AEISU_ERR_UNSUPPORTED);
    TcHostPack P;
    // Activation scales of the artifact times the model's power-of-two headroom (1 unless the
    // caller asked for more at load time: then the artifact's own quantisation points).  E4M3
    // is a floating point format, so a factor h leaves the rounding of every value below the
    // old limit bit-identical and only stops values in [448 s, 448 h s) from saturating (the
    // artifact was calibrated on natural images; high-contrast content exceeds its range in
    // the later bottleneck layers).
    // The INT8 route uses the artifact's scales as they are: int8 codes saturate at +-127 there
    // exactly as in the reference's kernels.
    float s[10];
    for (int i = 0; i < 10; ++i) s[i] = m.act_scales[i] * (i8 ? 1.0f : m.fp8_headroom);
    // one LeakyReLU slope for every activated layer (the tail is linear), in [0, 1] so that the
    // kernels may evaluate it as max(v, slope * v)
    P.slope = m.layers[kProject].slope[0];
    require(P.slope >= 0.f && P.slope <= 1.f, "activation slope outside [0, 1]", AEISU_ERR_UNSUPPORTED);
    for (int l = 0; l < kLayerCount; ++l)
        if (l != kTail)
            for (float v : m.layers[l].slope)
                require(v == P.slope, "the tensor-core routes need one activation slope for all layers",
                        AEISU_ERR_UNSUPPORTED);
    P.inv_s1 = (fp8 || i8) ? 1.0f / s[1] : 1.f;
    P.stencil = append_floats(P.floats, std::vector<float>(m.stencil, m.stencil + 24));

    // project_540: [32 out][32 in], K = torch input channel order (feature c*4 + phase)
    {
        const LayerWeights& L = m.layers[kProject];
        P.project = append_bytes(P.bytes, pack_operand(32, 32, 2, [&](int n, int k) { return L.w_fp16[n * 32 + k]; }));
        P.project_bias = append_floats(P.floats, L.bias);
    }
    // per-channel epilogue vectors; `perm` maps the packed output order to the torch channel
    auto epilogue = [&](TcHostLayer& out, const LayerWeights& L, int n, float s_in, float s_out, auto perm) {
        std::vector<float> scale(n), bias(n);
        for (int i = 0; i < n; ++i) {
            const int o = perm(i);
            scale[i] = fp8 ? s_in * L.w_scale[o] : i8 ? L.factor[o] : 1.f;
            bias[i] = fp8 ? L.bias_fp8[o] : L.bias[o];
        }
        out.scale = append_floats(P.floats, scale);
        out.bias = append_floats(P.floats, bias);
        out.out_inv = (fp8 || i8) ? 1.0f / s_out : 1.f;
    };
    const int es = fp8 ? 1 : 2;
    auto elem = [&](const LayerWeights& L, size_t idx) -> uint32_t { return fp8 ? L.w_fp8[idx] : L.w_fp16[idx]; };

    // compress_270: [64][128]; packed K order phase*32 + c <- torch input c*4 + phase
    {
        const LayerWeights& L = m.layers[kCompress];
        P.compress.image = append_bytes(P.bytes, pack_operand(64, 128, es, [&](int n, int kk) {
            return elem(L, size_t(n) * 128 + (kk % 32) * 4 + kk / 32);
        }));
        epilogue(P.compress, L, 64, s[1], s[2], [](int i) { return i; });
    }
    // bottleneck i: two groups of [32 out][9 taps x 32 in], chunks ordered [kx][chunk][ky] so
    // that the blocks of tap rows ky and ky+1 are adjacent and one N = 64 operand covers both
    for (int i = 0; i < 4; ++i) {
        const LayerWeights& L = m.layers[kCore0 + i];
        std::vector<uint8_t> img;
        const int epc = 16 / es, cpg = 32 / epc;   // elements per 16-byte chunk, chunks per tap
        for (int g = 0; g < 2; ++g) {
            auto part = pack_operand(32, 288, es, [&](int n, int kv) {
                const int c = kv / epc, ky = c % 3, kc = (c / 3) % cpg, kx = c / (3 * cpg);
                return elem(L, (size_t(g * 32 + n) * 32 + kc * epc + kv % epc) * 9 + ky * 3 + kx);
            });
            img.insert(img.end(), part.begin(), part.end());
        }
        P.core[i].image = append_bytes(P.bytes, img);
        epilogue(P.core[i], L, 64, s[i + 2], s[i + 3], [](int n) { return n; });
    }
    // expand_270: [128][64], output order phase*32 + c <- torch output c*4 + phase
    {
        const LayerWeights& L = m.layers[kExpand];
        auto torch_out = [](int n) { return (n % 32) * 4 + n / 32; };
        P.expand.image = append_bytes(P.bytes, pack_operand(128, 64, es, [&](int n, int k) {
            return elem(L, size_t(torch_out(n)) * 64 + k);
        }));
        epilogue(P.expand, L, 128, s[6], s[7], torch_out);
        P.expand.out_deq = (fp8 || i8) ? s[7] : 1.f;
    }
    // refine_540: [64][9 taps x 32] f16 in both routes, chunks ordered [kx][k4][ky] (k4: 8 input
    // channels) so that the blocks of tap rows ky and ky+1 are adjacent and one N = 128 operand
    // covers both; metadata_head [64][64] f16
    {
        const LayerWeights& R = m.layers[kRefine];
        P.refine = append_bytes(P.bytes, pack_operand(64, 288, 2, [&](int n, int kv) {
            const int c = kv / 8, ky = c % 3, k4 = (c / 3) % 4, kx = c / 12;
            return R.w_fp16[(size_t(n) * 32 + k4 * 8 + kv % 8) * 9 + ky * 3 + kx];
        }));
        P.refine_bias = append_floats(P.floats, R.bias);
        const LayerWeights& T = m.layers[kTail];
        P.tail = append_bytes(P.bytes, pack_operand(64, 64, 2, [&](int n, int k) { return T.w_fp16[n * 64 + k]; }));
        std::vector<float> tb(64);
        // f16 tail bias on the native routes (Refine.cuh:494-495); the INT8 route's finish adds
        // its FP32 bias (optimized/shader/runtime.py:221, finish_controller)
        for (int i = 0; i < 64; ++i) tb[i] = i8 ? T.bias[i] : round_f16(T.bias[i]);
        P.tail_bias = append_floats(P.floats, tb);
    }
    // head: 100 of 128 columns, FP32 bank split into hi + lo f16.  Columns 0..79 hold the
    // horizontally paired taps (ky, 2j) and (ky, 2j+1), j = 0, 1, as n = (ky*2 + j)*8 +
    // phase*2 + (kx & 1), so one packed f32x2 FMA applies both taps of a pair; columns 80..99
    // hold the fifth column's taps (ky, 4) as n = 80 + ky*4 + phase.
    {
        auto tap_phase = [](int n, int& tap, int& phase) {
            if (n < 80) {
                const int pair = n / 8;
                phase = (n / 2) % 4;
                tap = (pair / 2) * 5 + (pair % 2) * 2 + n % 2;
                return true;
            }
            if (n < 100) {
                phase = (n - 80) % 4;
                tap = ((n - 80) / 4) * 5 + 4;
                return true;
            }
            return false;
        };
        auto bank = [&](int n, int k, bool lo) -> uint32_t {
            int tap, phase;
            if (!tap_phase(n, tap, phase)) return 0;
            const float v = m.basis[(tap * 16 + k) * 4 + phase];
            const uint16_t hi = f32_to_f16_bits(v);
            return lo ? f32_to_f16_bits(v - f16_bits_to_f32(hi)) : hi;
        };
        auto hi = pack_operand(128, 16, 2, [&](int n, int k) { return bank(n, k, false); });
        auto lo = pack_operand(128, 16, 2, [&](int n, int k) { return bank(n, k, true); });
        auto base = pack_operand(128, 16, 2, [&](int n, int k) -> uint32_t {
            int tap, phase;
            if (!tap_phase(n, tap, phase) || k > 1) return 0;
            const float v = m.base[tap * 4 + phase];
            const uint16_t h = f32_to_f16_bits(v);
            return k == 0 ? h : f32_to_f16_bits(v - f16_bits_to_f32(h));
        });
        std::vector<uint8_t> img(hi);
        img.insert(img.end(), lo.begin(), lo.end());
        img.insert(img.end(), base.begin(), base.end());
        P.head = append_bytes(P.bytes, img);
    }
    while (P.bytes.size() % 128) P.bytes.push_back(0);
    return P;
}

}  // namespace aeisu
