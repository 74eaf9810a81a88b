// extern "C" boundary (include/aeisu.h).  Every entry point converts internal failures
// into status codes and records the message for aeisu_last_error().
#include <cmath>
#include <cstring>
#include <fstream>
#include <iterator>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "engine.h"
#include "kernels.h"
#include "model.h"
#include "noalloc.h"

struct aeisu_engine {
    std::unique_ptr<aeisu::Engine> engine;
};

namespace {

thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f) {
    try {
        f();
        g_last_error.clear();
        return AEISU_OK;
    } catch (const aeisu::Error& e) {
        g_last_error = e.what();
        return e.status;
    } catch (const std::bad_alloc&) {
        g_last_error = "host allocation failed";
        return AEISU_ERR_OOM;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return AEISU_ERR_INVALID_ARG;
    }
}

int open_model(aeisu::HostModel&& m, int precision, int device, aeisu_t** out) {
    aeisu::require(out != nullptr, "output handle pointer is null");
    *out = nullptr;
    auto h = std::make_unique<aeisu_engine>();
    h->engine = std::make_unique<aeisu::Engine>(std::move(m), precision, device);
    *out = h.release();
    return AEISU_OK;
}

aeisu::Engine& engine_of(aeisu_t* h) {
    aeisu::require(h != nullptr && h->engine != nullptr, "handle is null");
    return *h->engine;
}

void check_io(int n, int h, int w, unsigned flags) {
    aeisu::require(n >= 1 && h >= 1 && w >= 1, "Expected CHW RGB image");
    aeisu::require(flags == AEISU_IO_HOST || flags == AEISU_IO_DEVICE, "unknown I/O flags");
}

}  // namespace

extern "C" {

int aeisu_validate_spyr8(const void* data, size_t bytes, char* checksum_hex) {
    return guarded([&] {
        aeisu::HostModel m = aeisu::load_spyr8(static_cast<const uint8_t*>(data), bytes);
        if (checksum_hex) {
            std::memcpy(checksum_hex, m.checksum_hex.c_str(), 64);
            checksum_hex[64] = 0;
        }
    });
}

int aeisu_open_spyr8_memory(const void* data, size_t bytes, int precision, int device, aeisu_t** out) {
    return guarded([&] {
        aeisu::HostModel m = aeisu::load_spyr8(static_cast<const uint8_t*>(data), bytes);
        open_model(std::move(m), precision, device, out);
    });
}

int aeisu_open_spyr8_headroom(const void* data, size_t bytes, int precision, int device,
                              float activation_headroom, aeisu_t** out) {
    return guarded([&] {
        const float h = activation_headroom;
        int e = 0;
        aeisu::require(h >= 1.f && h <= 64.f && std::frexp(h, &e) == 0.5f,
                       "activation headroom must be a power of two in [1, 64]");
        aeisu::HostModel m = aeisu::load_spyr8(static_cast<const uint8_t*>(data), bytes);
        m.fp8_headroom = h;
        open_model(std::move(m), precision, device, out);
    });
}

int aeisu_open_spyr8(const char* path, int precision, int device, aeisu_t** out) {
    return guarded([&] {
        aeisu::require(path != nullptr, "path is null");
        std::ifstream f(path, std::ios::binary);
        if (!f) aeisu::fail(AEISU_ERR_BAD_ARTIFACT, std::string("could not open SPYR8 model: ") + path);
        std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
        aeisu::HostModel m = aeisu::load_spyr8(reinterpret_cast<const uint8_t*>(bytes.data()), bytes.size());
        open_model(std::move(m), precision, device, out);
    });
}

int aeisu_open_int8(const aeisu_int8_artifact* artifact, int device, aeisu_t** out) {
    return guarded([&] {
        aeisu::require(out != nullptr, "output handle pointer is null");
        *out = nullptr;
        aeisu::require(artifact != nullptr, "artifact pointer is null");
        aeisu::HostModel m = aeisu::load_int8(*artifact);
        open_model(std::move(m), AEISU_PRECISION_INT8, device, out);
    });
}

int aeisu_open_folded(const float* values, size_t count, float basis_l1_scale, int precision, int device,
                      aeisu_t** out) {
    return guarded([&] {
        if (precision == AEISU_PRECISION_MIXED)
            aeisu::fail(AEISU_ERR_UNSUPPORTED, "MIXED precision needs the FP8 scales of a SPYR8 artifact");
        aeisu::HostModel m = aeisu::load_folded(values, count, basis_l1_scale);
        open_model(std::move(m), precision, device, out);
    });
}

int aeisu_open_sibling(aeisu_t* handle, aeisu_t** out) {
    return guarded([&] {
        aeisu::require(out != nullptr, "output handle pointer is null");
        *out = nullptr;
        const aeisu::Engine& parent = engine_of(handle);
        auto h = std::make_unique<aeisu_engine>();
        h->engine = std::make_unique<aeisu::Engine>(parent, aeisu::Engine::Sibling{});
        *out = h.release();
    });
}

void aeisu_close(aeisu_t* handle) { delete handle; }

int aeisu_upscale_u8(aeisu_t* handle, const uint8_t* src, int n, int h, int w, int tile, uint8_t* dst,
                     unsigned flags, void* stream) {
    return guarded([&] {
        check_io(n, h, w, flags);
        aeisu::Call c{aeisu::Mode::Upscale, src, 0, dst, 0, n, h, w, tile, flags == AEISU_IO_HOST,
                      static_cast<cudaStream_t>(stream)};
        engine_of(handle).run(c);
    });
}

int aeisu_upscale_u8_band(aeisu_t* handle, const uint8_t* src, int h, int w, int band, int bands, uint8_t* dst,
                          unsigned flags, void* stream) {
    return guarded([&] {
        check_io(1, h, w, flags);
        aeisu::Call c{aeisu::Mode::Upscale, src, 0, dst, 0, 1, h, w, 0, flags == AEISU_IO_HOST,
                      static_cast<cudaStream_t>(stream)};
        c.band = band;
        c.bands = bands;
        aeisu::require(bands >= 1 && band >= 0 && band < bands, "band index out of range");
        engine_of(handle).run(c);
    });
}

int aeisu_upscale_u8_noalloc(aeisu_t* handle, const uint8_t* src, int n, int h, int w, uint8_t* dst,
                             void* stream) {
    return guarded([&] {
        aeisu::upscale_u8_noalloc(engine_of(handle), src, n, h, w, dst, static_cast<cudaStream_t>(stream));
    });
}

int aeisu_upscale_f32(aeisu_t* handle, const float* src, int n, int h, int w, int tile, float* dst,
                      unsigned flags, void* stream) {
    return guarded([&] {
        check_io(n, h, w, flags);
        aeisu::Call c{aeisu::Mode::Upscale, src, 1, dst, 1, n, h, w, tile, flags == AEISU_IO_HOST,
                      static_cast<cudaStream_t>(stream)};
        engine_of(handle).run(c);
    });
}

int aeisu_forward_f32(aeisu_t* handle, const float* src, int n, int h, int w, float* dst, unsigned flags,
                      void* stream) {
    return guarded([&] {
        check_io(n, h, w, flags);
        aeisu::Call c{aeisu::Mode::Forward, src, 1, dst, 1, n, h, w, 0, flags == AEISU_IO_HOST,
                      static_cast<cudaStream_t>(stream)};
        engine_of(handle).run(c);
    });
}

int aeisu_predict_coefficients(aeisu_t* handle, const float* src, int n, int h, int w, float* meta,
                               unsigned flags, void* stream) {
    return guarded([&] {
        check_io(n, h, w, flags);
        aeisu::Call c{aeisu::Mode::Predict, src, 1, meta, 1, n, h, w, 0, flags == AEISU_IO_HOST,
                      static_cast<cudaStream_t>(stream)};
        engine_of(handle).run(c);
    });
}

int aeisu_activation_stats(aeisu_t* handle, const uint8_t* src, int n, int h, int w, unsigned flags, float* peaks,
                           float* means, void* stream) {
    return guarded([&] {
        check_io(n, h, w, flags);
        engine_of(handle).activation_stats(src, flags == AEISU_IO_HOST, n, h, w, peaks, means,
                                           static_cast<cudaStream_t>(stream));
    });
}

int aeisu_distortion(const float* prediction, const float* target, int n, int h, int w, int crop, unsigned flags,
                     int device, double* out, void* stream) {
    return guarded([&] {
        aeisu::require(flags == AEISU_IO_HOST || flags == AEISU_IO_DEVICE, "unknown I/O flags");
        aeisu::distortion(prediction, target, n, h, w, crop, flags == AEISU_IO_HOST, device, out,
                          static_cast<cudaStream_t>(stream));
    });
}

uint64_t aeisu_png_bound(int h, int w) {
    uint64_t r = 0;
    const int st = guarded([&] { r = aeisu::png_bound(h, w); });
    return st == AEISU_OK ? r : 0;
}

int aeisu_png_encode(const void* frames, int kind, int n, int h, int w, unsigned flags, int device, uint8_t* out,
                     uint64_t capacity, uint64_t* sizes, void* stream) {
    return guarded([&] {
        aeisu::require(flags == AEISU_IO_HOST || flags == AEISU_IO_DEVICE, "unknown I/O flags");
        aeisu::png_encode(frames, kind, n, h, w, flags == AEISU_IO_HOST, device, out, capacity, sizes,
                          static_cast<cudaStream_t>(stream));
    });
}

int aeisu_png_info(const uint8_t* file, uint64_t bytes, int* h, int* w, int* color_type) {
    return guarded([&] {
        aeisu::require(h && w && color_type, "output pointers are null");
        const aeisu::PngFileInfo info = aeisu::png_parse(file, size_t(bytes), nullptr);
        aeisu::png_check_supported(info);
        *h = info.h;
        *w = info.w;
        *color_type = info.color;
    });
}

int aeisu_png_decode(const uint8_t* files, const uint64_t* offsets, const uint64_t* sizes, int n, int h, int w,
                     unsigned flags, int device, uint8_t* out, void* stream) {
    return guarded([&] {
        aeisu::require(flags == AEISU_IO_HOST || flags == AEISU_IO_DEVICE, "unknown I/O flags");
        aeisu::png_decode(files, offsets, sizes, n, h, w, flags == AEISU_IO_HOST, device, out,
                          static_cast<cudaStream_t>(stream));
    });
}

int aeisu_reconstruct_f32(const float* source, const float* metadata, const float* base, const float* basis, int n,
                          int h, int w, int trim, int device, float* out, void* stream) {
    return guarded([&] {
        aeisu::reconstruct_f32(source, metadata, base, basis, n, h, w, trim, device, out,
                               static_cast<cudaStream_t>(stream));
    });
}

int aeisu_reconstruct_backward_f32(const float* source, const float* metadata, const float* basis,
                                   const float* grad_out, int n, int h, int w, int trim, int gradient_stride,
                                   int phase, int device, float* grad_metadata, float* grad_base,
                                   float* grad_basis, void* stream) {
    return guarded([&] {
        aeisu::reconstruct_backward_f32(source, metadata, basis, grad_out, n, h, w, trim, gradient_stride, phase,
                                        device, grad_metadata, grad_base, grad_basis,
                                        static_cast<cudaStream_t>(stream));
    });
}

int aeisu_tensor_peak(int device, int kind, int ctas_per_sm, int mmas_per_cta, int repeats, double* tflops) {
    return guarded([&] {
        aeisu::require(tflops != nullptr, "tflops pointer is null");
        *tflops = aeisu::tensor_peak_tflops(device, kind, ctas_per_sm, mmas_per_cta, repeats);
    });
}

int aeisu_synchronize(aeisu_t* handle, void* stream, double timeout_ms) {
    return guarded([&] { engine_of(handle).synchronize(static_cast<cudaStream_t>(stream), timeout_ms); });
}

int aeisu_timings_get(aeisu_t* handle, aeisu_timings* out) {
    return guarded([&] {
        aeisu::require(out != nullptr, "timings pointer is null");
        *out = engine_of(handle).timings();
    });
}

int aeisu_set_detailed_timing(aeisu_t* handle, int enabled) {
    return guarded([&] { engine_of(handle).set_detailed(enabled != 0); });
}

int aeisu_set_fused_head(aeisu_t* handle, int enabled) {
    return guarded([&] { engine_of(handle).set_fused_head(enabled != 0); });
}

int aeisu_set_workspace_limit(aeisu_t* handle, uint64_t bytes) {
    return guarded([&] { engine_of(handle).set_workspace_cap(size_t(bytes)); });
}

int aeisu_set_timeout(aeisu_t* handle, double timeout_ms) {
    return guarded([&] {
        aeisu::require(timeout_ms > 0, "timeout must be positive");
        engine_of(handle).set_timeout(timeout_ms);
    });
}

const char* aeisu_report(aeisu_t* handle) {
    if (!handle || !handle->engine) return "";
    return handle->engine->report().c_str();
}

uint64_t aeisu_device_bytes(aeisu_t* handle) {
    return (handle && handle->engine) ? handle->engine->device_bytes() : 0;
}

uint64_t aeisu_kernel_launches(aeisu_t* handle) {
    return (handle && handle->engine) ? handle->engine->launches() : 0;
}

const char* aeisu_last_error(void) { return g_last_error.c_str(); }

const char* aeisu_version(void) { return "aeisu-b200 0.1.0 (sm_100a)"; }

}  // extern "C"
