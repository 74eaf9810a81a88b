// Engine: owns one model on one GPU and runs inference calls.  Padding and tiling follow
// aeisu/runtime.py:70-103; the launch sequence per region batch follows the reference's
// mixed frame body (optimized/native/src/neural/srcpyr/SrcPyrCudaRuntime.cu:4131-4873):
// analysis+project -> compress+core -> expand+shuffle+skip -> refine+tail -> head.
#include "engine.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <map>
#include <sstream>
#include <thread>

#include "common.h"
#include "tc_pack.h"

namespace aeisu {

DevBuf::~DevBuf() { reset(); }

void DevBuf::reset() {
    if (p_) cudaFree(p_);
    p_ = nullptr;
    cap_ = 0;
}

void* DevBuf::ensure(size_t bytes, cudaStream_t s) {
    if (bytes <= cap_) return p_;
    if (p_) {
        AEISU_CUDA(cudaStreamSynchronize(s));
        AEISU_CUDA(cudaFree(p_));
        p_ = nullptr;
        cap_ = 0;
    }
    bytes = (bytes + 255) / 256 * 256;
    AEISU_CUDA(cudaMalloc(&p_, bytes));
    cap_ = bytes;
    return p_;
}

void HostBuf::reset() {
    if (p_) cudaFreeHost(p_);
    p_ = nullptr;
    cap_ = 0;
}

void* HostBuf::ensure(size_t bytes, cudaStream_t s) {
    if (bytes <= cap_) return p_;
    if (p_) {
        AEISU_CUDA(cudaStreamSynchronize(s));
        reset();
    }
    AEISU_CUDA(cudaHostAlloc(&p_, bytes, cudaHostAllocDefault));
    cap_ = bytes;
    return p_;
}

namespace {
// True when `p` is page-locked (or otherwise directly DMA-able) host memory.
bool is_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}
}  // namespace

// ---- geometry -----------------------------------------------------------------------

Geometry plan_upscale(int n, int h, int w, int tile) {
    require(n >= 1 && h >= 1 && w >= 1, "frame count and size must be positive");
    require(tile >= 0 && tile % 32 == 0, "tile must be zero or a positive multiple of 32");
    require(int64_t(h) * w <= (int64_t(1) << 28) && h <= 32768 && w <= 32768, "frame too large");
    Geometry g{};
    g.n = n; g.h = h; g.w = w;
    const int ey = (32 - h % 32) % 32, ex = (32 - w % 32) % 32;   // -h % 32 in Python
    g.pad_y = 16 + ey / 2;
    g.pad_x = 16 + ex / 2;
    g.ph = h + 32 + ey;
    g.pw = w + 32 + ex;
    g.out_h = h; g.out_w = w;
    std::map<std::pair<int, int>, size_t> index;
    auto add = [&](const Region& r, int rh, int rw) {
        auto key = std::make_pair(rh, rw);
        auto it = index.find(key);
        if (it == index.end()) {
            index[key] = g.groups.size();
            g.groups.push_back({rh, rw, {}});
            it = index.find(key);
        }
        g.groups[it->second].regions.push_back(r);
    };
    for (int f = 0; f < n; ++f) {
        if (tile == 0) {
            add({f, 0, 0, g.pad_y, g.pad_x, g.pad_y + h, g.pad_x + w}, g.ph, g.pw);
            continue;
        }
        for (int y = 0; y < g.ph; y += tile)
            for (int x = 0; x < g.pw; x += tile) {
                const int y1 = std::min(y + tile, g.ph), x1 = std::min(x + tile, g.pw);
                const int sy = std::max(0, y - 32), sx = std::max(0, x - 32);
                const int ey2 = std::min(g.ph, y1 + 32), ex2 = std::min(g.pw, x1 + 32);
                // LR rows/cols of this core that survive the final crop (runtime.py:100)
                const int cy0 = std::max(y, g.pad_y), cy1 = std::min(y1, g.pad_y + h);
                const int cx0 = std::max(x, g.pad_x), cx1 = std::min(x1, g.pad_x + w);
                if (cy0 >= cy1 || cx0 >= cx1) continue;
                add({f, sy, sx, cy0 - sy, cx0 - sx, cy1 - sy, cx1 - sx}, ey2 - sy, ex2 - sx);
            }
    }
    return g;
}

Geometry plan_whole(int n, int h, int w) {
    require(n >= 1 && h >= 4 && w >= 4, "frame count and size must be positive");
    require(h % 4 == 0 && w % 4 == 0, "Source H/W must be divisible by 4");
    require(int64_t(h) * w <= (int64_t(1) << 28), "frame too large");
    Geometry g{};
    g.n = n; g.h = h; g.w = w;
    g.pad_y = g.pad_x = 0;
    g.ph = h; g.pw = w;
    g.out_h = h; g.out_w = w;
    g.groups.push_back({h, w, {}});
    for (int f = 0; f < n; ++f) g.groups[0].regions.push_back({f, 0, 0, 0, 0, h, w});
    return g;
}

Geometry plan_band(int h, int w, int band, int bands) {
    require(bands >= 1 && bands <= 4096 && band >= 0 && band < bands, "band index out of range");
    Geometry g = plan_upscale(1, h, w, 0);
    g.groups.clear();
    const int per = (g.ph / 32 + bands - 1) / bands * 32;
    const int y = band * per, y1 = std::min(g.ph, y + per);
    if (y >= y1) return g;   // more bands than 32-row groups: nothing left for this one
    const int sy = std::max(0, y - 32), ey = std::min(g.ph, y1 + 32);
    const int cy0 = std::max(y, g.pad_y), cy1 = std::min(y1, g.pad_y + h);
    if (cy0 < cy1) g.groups.push_back({ey - sy, g.pw, {{0, sy, 0, cy0 - sy, g.pad_x, cy1 - sy, g.pad_x + w}}});
    return g;
}

// ---- engine -------------------------------------------------------------------------

struct Engine::DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        AEISU_CUDA(cudaGetDevice(&prev));
        if (prev != dev) AEISU_CUDA(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
    }
};

Engine::Engine(HostModel model, int precision, int device)
    : model_(std::move(model)), precision_(precision), device_(device) {
    require(precision >= AEISU_PRECISION_FP32 && precision <= AEISU_PRECISION_INT8, "unknown precision");
    int count = 0;
    AEISU_CUDA(cudaGetDeviceCount(&count));
    require(device >= 0 && device < count, "device index out of range");
    if (precision == AEISU_PRECISION_MIXED && !model_.has_fp8)
        fail(AEISU_ERR_UNSUPPORTED, "MIXED precision needs the FP8 weights and scales of a SPYR8 artifact");
    if ((precision == AEISU_PRECISION_INT8) != model_.has_int8)
        fail(AEISU_ERR_UNSUPPORTED, model_.has_int8 ? "the INT8 artifact runs only at INT8 precision"
                                                    : "INT8 precision needs the INT8/FP16 artifact (aeisu_open_int8)");
    DeviceGuard guard(device_);
    cudaDeviceProp dp{};
    AEISU_CUDA(cudaGetDeviceProperties(&dp, device_));
    if (precision != AEISU_PRECISION_FP32 && !(dp.major == 10 && dp.minor == 0))
        fail(AEISU_ERR_UNSUPPORTED, "the tensor-core routes need an sm_100 (B200) device");
    create_streams();
    upload_weights();
    cudaDeviceProp prop{};
    AEISU_CUDA(cudaGetDeviceProperties(&prop, device_));
    std::ostringstream os;
    os << "aeisu-b200: device " << device_ << " " << prop.name << " (sm_" << prop.major << prop.minor << ", "
       << prop.multiProcessorCount << " SMs); model " << model_.format << " " << model_.architecture;
    if (!model_.checksum_hex.empty()) os << " sha256 " << model_.checksum_hex;
    os << "; precision " << (precision_ == 0 ? "fp32" : precision_ == 1 ? "fp16" : precision_ == 2 ? "mixed" : "int8");
    if (precision_ == AEISU_PRECISION_FP32) os << "; route simt-fp32 controller + fp32 head";
    else if (precision_ == AEISU_PRECISION_FP16) os << "; route tcgen05 f16 controller + tcgen05 head";
    else if (precision_ == AEISU_PRECISION_INT8)
        os << "; route tcgen05 int8-code/f16 controller (codes as f16, exact integer sums) + tcgen05 head";
    else os << "; route tcgen05 e4m3/f16 mixed controller + tcgen05 head; activation headroom x" << model_.fp8_headroom;
    report_ = os.str();
}

void Engine::create_streams() {
    int lo = 0, hi = 0;
    AEISU_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    AEISU_CUDA(cudaStreamCreateWithPriority(&stream_, cudaStreamNonBlocking, hi));
    AEISU_CUDA(cudaStreamCreateWithFlags(&copy_in_, cudaStreamNonBlocking));
    AEISU_CUDA(cudaStreamCreateWithFlags(&copy_out_, cudaStreamNonBlocking));
    AEISU_CUDA(cudaStreamCreateWithPriority(&lane_, cudaStreamNonBlocking, hi));
    AEISU_CUDA(cudaEventCreateWithFlags(&fork_, cudaEventDisableTiming));
    AEISU_CUDA(cudaEventCreateWithFlags(&join_, cudaEventDisableTiming));
    for (auto& e : ev_) AEISU_CUDA(cudaEventCreate(&e));
    flag_.ensure(256, stream_);
    AEISU_CUDA(cudaMemset(flag_.get(), 0, 256));
}

Engine::Engine(const Engine& parent, Sibling)
    : model_(parent.model_), precision_(parent.precision_), device_(parent.device_), report_(parent.report_),
      timeout_ms_(parent.timeout_ms_), weights_(parent.weights_), stencil_(parent.stencil_), base_(parent.base_),
      basis_(parent.basis_), tcw_(parent.tcw_), head_img_(parent.head_img_), workspace_cap_(parent.workspace_cap_) {
    for (int l = 0; l < kLayerCount; ++l) f32_layers_[l] = parent.f32_layers_[l];
    DeviceGuard guard(device_);
    create_streams();
    report_ += "; sibling handle (shared weights)";
}

Engine::~Engine() {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (cudaStream_t c : {copy_in_, copy_out_, lane_})
        if (c) cudaStreamSynchronize(c);
    DevBuf* all[] = {&src_, &dst_, &tables_, &flag_, &stats_};
    for (DevBuf* b : all) b->reset();
    for (Workspace& w : ws_)
        for (DevBuf* b : {&w.enc540, &w.low_a, &w.low_b, &w.dec540, &w.refined, &w.meta, &w.encu, &w.raw}) b->reset();
    weights_.reset();   // freed here when this is the last handle sharing them
    table_cache_.clear();
    staging_.reset();
    for (auto& e : ev_)
        if (e) cudaEventDestroy(e);
    for (auto& e : pool_) cudaEventDestroy(e);
    for (auto& e : chunk_ev_) cudaEventDestroy(e);
    if (stream_) cudaStreamDestroy(stream_);
    for (cudaStream_t c : {copy_in_, copy_out_, lane_})
        if (c) cudaStreamDestroy(c);
    for (cudaEvent_t e : {fork_, join_})
        if (e) cudaEventDestroy(e);
    if (prev >= 0) cudaSetDevice(prev);
}

uint64_t Engine::device_bytes() const {
    const DevBuf* all[] = {&src_, &dst_, &tables_, &flag_, &stats_, &weights_->w_f32, &weights_->tc_bytes,
                           &weights_->tc_floats};
    uint64_t total = 0;
    for (auto* b : all) total += b->capacity();
    for (const Workspace& w : ws_)
        for (const DevBuf* b : {&w.enc540, &w.low_a, &w.low_b, &w.dec540, &w.refined, &w.meta, &w.encu, &w.raw})
            total += b->capacity();
    return total;
}

void Engine::upload_weights() {
    // FP32 tensors packed in one allocation: stencil, base, basis, then per layer w | b.
    std::vector<float> host;
    auto push = [&](const float* p, size_t n) {
        size_t at = host.size();
        host.insert(host.end(), p, p + n);
        while (host.size() % 64) host.push_back(0.f);
        return at;
    };
    const size_t o_st = push(model_.stencil, 24);
    const size_t o_base = push(model_.base, 100);
    const size_t o_basis = push(model_.basis, 1600);
    size_t o_w[kLayerCount], o_b[kLayerCount];
    for (int l = 0; l < kLayerCount; ++l) {
        const LayerWeights& L = model_.layers[l];
        o_w[l] = push(L.w.data(), L.w.size());
        o_b[l] = push(L.bias.data(), L.bias.size());
        for (float s : L.slope)
            if (s != L.slope[0]) fail(AEISU_ERR_UNSUPPORTED, "per-channel activation slopes are not supported");
    }
    weights_ = std::make_shared<ResidentWeights>();
    DevBuf& w_f32 = weights_->w_f32;
    w_f32.ensure(host.size() * 4, stream_);
    AEISU_CUDA(cudaMemcpy(w_f32.get(), host.data(), host.size() * 4, cudaMemcpyHostToDevice));
    const float* d = w_f32.as<float>();
    stencil_ = d + o_st;
    base_ = d + o_base;
    basis_ = d + o_basis;
    for (int l = 0; l < kLayerCount; ++l)
        f32_layers_[l] = {d + o_w[l], d + o_b[l], model_.layers[l].slope[0]};
    if (precision_ == AEISU_PRECISION_FP32) return;
    const TcHostPack P = pack_tc(model_, tc_route_of(precision_));
    DevBuf& tc_bytes = weights_->tc_bytes;
    DevBuf& tc_floats = weights_->tc_floats;
    tc_bytes.ensure(P.bytes.size(), stream_);
    tc_floats.ensure(P.floats.size() * 4, stream_);
    AEISU_CUDA(cudaMemcpy(tc_bytes.get(), P.bytes.data(), P.bytes.size(), cudaMemcpyHostToDevice));
    AEISU_CUDA(cudaMemcpy(tc_floats.get(), P.floats.data(), P.floats.size() * 4, cudaMemcpyHostToDevice));
    const uint8_t* B = tc_bytes.as<uint8_t>();
    const float* F = tc_floats.as<float>();
    auto ep = [&](const TcHostLayer& L) { return EpiParams{P.slope, L.out_inv, L.out_deq}; };
    std::copy(P.floats.begin() + P.stencil, P.floats.begin() + P.stencil + 24, tcw_.proj.st);
    std::copy(P.floats.begin() + P.project_bias, P.floats.begin() + P.project_bias + 32, tcw_.proj.bias);
    tcw_.project = B + P.project;
    tcw_.slope = P.slope;
    tcw_.inv_s1 = P.inv_s1;
    tcw_.compress = B + P.compress.image;
    tcw_.compress_ep = ep(P.compress);
    std::copy(P.floats.begin() + P.compress.scale, P.floats.begin() + P.compress.scale + 64, tcw_.compress_cp.scale);
    std::copy(P.floats.begin() + P.compress.bias, P.floats.begin() + P.compress.bias + 64, tcw_.compress_cp.bias);
    for (int i = 0; i < 4; ++i) {
        tcw_.core[i] = B + P.core[i].image;
        tcw_.core_ep[i] = ep(P.core[i]);
        std::copy(P.floats.begin() + P.core[i].scale, P.floats.begin() + P.core[i].scale + 64, tcw_.core_cp[i].scale);
        std::copy(P.floats.begin() + P.core[i].bias, P.floats.begin() + P.core[i].bias + 64, tcw_.core_cp[i].bias);
    }
    tcw_.expand = B + P.expand.image;
    tcw_.expand_ep = ep(P.expand);
    std::copy(P.floats.begin() + P.expand.scale, P.floats.begin() + P.expand.scale + 128, tcw_.expand_cp.scale);
    std::copy(P.floats.begin() + P.expand.bias, P.floats.begin() + P.expand.bias + 128, tcw_.expand_cp.bias);
    tcw_.refine = B + P.refine;
    tcw_.tail = B + P.tail;
    tcw_.refine_bias = F + P.refine_bias;
    tcw_.tail_bias = F + P.tail_bias;
    std::copy(P.floats.begin() + P.refine_bias, P.floats.begin() + P.refine_bias + 64, tcw_.rbias.refine);
    std::copy(P.floats.begin() + P.tail_bias, P.floats.begin() + P.tail_bias + 64, tcw_.rbias.tail);
    tcw_.head = B + P.head;
    head_img_ = B + P.head;
}

void Engine::record(int stage, cudaStream_t s) {
    if (!detailed_) return;
    // Stage marks are events recorded in stream order without waiting; timings() resolves
    // them once the work has completed.  Mark i closes stage marks_[i].first.
    if (marks_.size() == pool_.size()) {
        cudaEvent_t e;
        AEISU_CUDA(cudaEventCreate(&e));
        pool_.push_back(e);
    }
    const size_t i = marks_.size();
    AEISU_CUDA(cudaEventRecord(pool_[i], s));
    marks_.push_back({stage, int(i)});
}

const aeisu_timings& Engine::timings() {
    if (!timings_pending_) return timings_;
    DeviceGuard guard(device_);
    AEISU_CUDA(cudaEventSynchronize(ev_[6]));
    timings_ = {};
    float per[6] = {};
    for (size_t i = 1; i < marks_.size(); ++i) {
        float ms = 0.f;
        AEISU_CUDA(cudaEventElapsedTime(&ms, pool_[marks_[i - 1].second], pool_[marks_[i].second]));
        if (marks_[i].first >= 1 && marks_[i].first <= 5) per[marks_[i].first] += ms;
    }
    timings_.analysis_project_ms = per[1];
    timings_.compress_core_ms = per[2];
    timings_.expand_ms = per[3];
    timings_.refine_tail_ms = per[4];
    timings_.reconstruction_ms = per[5];
    float total = 0.f;
    AEISU_CUDA(cudaEventElapsedTime(&total, ev_[0], ev_[6]));
    timings_.total_ms = total;
    timings_.detailed = marks_.size() > 1 ? 1 : 0;
    timings_pending_ = false;
    return timings_;
}

void Engine::wait(cudaStream_t s, double timeout_ms) {
    AEISU_CUDA(cudaEventRecord(ev_[7], s));
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaEventQuery(ev_[7]);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) AEISU_CUDA(e);
        const double el = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (el > timeout_ms)
            fail(AEISU_ERR_TIMEOUT, "GPU work did not complete within " + std::to_string(timeout_ms) + " ms");
        std::this_thread::sleep_for(std::chrono::microseconds(el < 5.0 ? 10 : 200));
    }
}

void Engine::synchronize(cudaStream_t s, double timeout_ms) {
    DeviceGuard guard(device_);
    if (!s) s = stream_;
    wait(s, timeout_ms);
    int flag[2] = {0, 0};
    AEISU_CUDA(cudaMemcpy(flag, flag_.get(), sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag[0] || flag[1]) AEISU_CUDA(cudaMemset(flag_.get(), 0, sizeof(flag)));
    if (flag[1]) fail(AEISU_ERR_CUDA, "tensor-core pipeline wait expired inside a kernel");
    if (flag[0]) fail(AEISU_ERR_NONFINITE, "Non-finite model reconstruction");
}

namespace {

struct RegionBytes {
    size_t enc, encu, low, dec, ref, meta, raw;
    size_t per_region() const { return enc + encu + 2 * low + dec + ref + meta + raw; }
};

// Workspace bytes per region: f32 NHWC for the FP32 route; chunk-planar f16/e4m3 otherwise.
// A fused tensor-core reconstruction keeps the coefficients on chip: no meta buffer.
RegionBytes region_bytes(int precision, int rh, int rw, bool predict, bool fused) {
    const size_t packed = size_t(rh / 2) * (rw / 2), low = size_t(rh / 4) * (rw / 4);
    const bool tcr = precision != AEISU_PRECISION_FP32, fp8 = precision == AEISU_PRECISION_MIXED;
    RegionBytes b;
    b.enc = tcr ? packed * 64 : packed * 32 * 4;
    b.encu = tcr ? low * (fp8 ? 128 : 256) : 0;
    b.low = tcr ? low * (fp8 ? 64 : 128) : low * 64 * 4;
    b.dec = tcr ? packed * 64 : packed * 32 * 4;
    b.ref = tcr ? 0 : packed * 64 * 4;
    b.meta = tcr ? (fused ? 0 : size_t(rh) * rw * 32) : packed * 64 * 4;
    b.raw = (tcr && predict) ? packed * 64 * 4 : 0;
    return b;
}

// Regions per batch from which a batch is split across two streams: below it the halves
// are too small to gain from overlapping (measured +4.7% at 64 frames of 1280x720).
constexpr int kSplitRegions = 8;

}  // namespace

void Engine::run_group(const Call& c, const Geometry& g, const Geometry::Group& grp, const SrcDesc& src,
                       const DstDesc& dst, cudaStream_t s) {
    const RegionBytes rb = region_bytes(precision_, grp.rh, grp.rw, c.mode == Mode::Predict, fused(c));
    const size_t chunk = std::max<size_t>(1, std::min<size_t>(grp.regions.size(), workspace_cap_ / rb.per_region()));
    for (size_t first = 0; first < grp.regions.size(); first += chunk) {
        const int R = int(std::min(chunk, grp.regions.size() - first));
        // Two halves on two streams: upscale calls of the tensor-core routes with enough regions,
        // unless the stage split is being timed (its marks are recorded on one stream).
        const bool split = precision_ != AEISU_PRECISION_FP32 && c.mode == Mode::Upscale && !detailed_ &&
                           R >= kSplitRegions;
        if (!split) {
            run_regions(c, grp, first, R, src, dst, s, ws_[0]);
            continue;
        }
        const int R0 = (R + 1) / 2;
        AEISU_CUDA(cudaEventRecord(fork_, s));
        AEISU_CUDA(cudaStreamWaitEvent(lane_, fork_, 0));
        run_regions(c, grp, first, R0, src, dst, s, ws_[0]);
        run_regions(c, grp, first + R0, R - R0, src, dst, lane_, ws_[1]);
        AEISU_CUDA(cudaEventRecord(join_, lane_));
        AEISU_CUDA(cudaStreamWaitEvent(s, join_, 0));
    }
    (void)g;
}

void Engine::run_regions(const Call& c, const Geometry::Group& grp, size_t first, int R, const SrcDesc& src,
                         const DstDesc& dst, cudaStream_t s, Workspace& ws) {
    const int rh = grp.rh, rw = grp.rw;
    const size_t packed = size_t(rh / 2) * (rw / 2);
    const bool tcr = precision_ != AEISU_PRECISION_FP32;
    const bool fuse = fused(c);
    const RegionBytes rb = region_bytes(precision_, rh, rw, c.mode == Mode::Predict, fuse);
    std::vector<int4> table(2 * size_t(R));
    int core_h = 0, core_w = 0;
    for (int i = 0; i < R; ++i) {
        const Region& r = grp.regions[first + i];
        table[i] = make_int4(r.frame, r.oy, r.ox, 0);
        table[R + i] = make_int4(r.cy0, r.cx0, r.cy1, r.cx1);
        core_h = std::max(core_h, r.cy1 - r.cy0);
        core_w = std::max(core_w, r.cx1 - r.cx0);
    }
    // Region tables are uploaded once per call geometry and kept on the device: an upload
    // from pageable memory would wait for the stream to drain on every call.
    const TableKey key{int(c.mode), c.n, c.h, c.w, c.tile, rh * 65536 + rw, int(first), R, c.band, c.bands};
    auto it = table_cache_.find(key);
    if (it == table_cache_.end()) {
        if (table_cache_.size() >= 256) {
            AEISU_CUDA(cudaDeviceSynchronize());
            table_cache_.clear();
        }
        auto buf = std::make_unique<DevBuf>();
        buf->ensure(table.size() * sizeof(int4), s);
        AEISU_CUDA(cudaMemcpy(buf->get(), table.data(), table.size() * sizeof(int4), cudaMemcpyHostToDevice));
        it = table_cache_.emplace(key, std::move(buf)).first;
    }
    RegionSet rs{};
    rs.regions = it->second->as<int4>();
    rs.cores = it->second->as<int4>() + R;
    rs.R = R; rs.rh = rh; rs.rw = rw; rs.core_h = core_h; rs.core_w = core_w;
    ws.enc540.ensure(rb.enc * R, s);
    ws.dec540.ensure(rb.dec * R, s);
    if (rb.ref) ws.refined.ensure(rb.ref * R, s);
    if (rb.encu) ws.encu.ensure(rb.encu * R, s);
    if (rb.raw) ws.raw.ensure(rb.raw * R, s);
    if (rb.meta) ws.meta.ensure(rb.meta * R, s);
    ws.low_a.ensure(rb.low * R, s);
    ws.low_b.ensure(rb.low * R, s);
    int launches = 0;
    struct Ctx { Engine* e; cudaStream_t s; } ctx{this, s};
    StageMark mark;
    mark.ctx = &ctx;
    mark.fn = [](void* p, int stage) { auto* c = static_cast<Ctx*>(p); c->e->record(stage, c->s); };
    const bool predict = c.mode == Mode::Predict;
    if (tcr) {
        const FusedHead head{&dst, head_img_, flag_.as<int>()};
        launch_tc_controller(tc_route_of(precision_), src, rs, tcw_, ws.enc540.get(), ws.encu.get(), ws.low_a.get(),
                             ws.low_b.get(), ws.dec540.get(), ws.meta.get(), predict ? ws.raw.as<float>() : nullptr,
                             flag_.as<int>() + 1, s, &launches, mark, fuse ? &head : nullptr);
    } else {
        launch_f32_controller(src, rs, stencil_, f32_layers_, ws.enc540.as<float>(), ws.low_a.as<float>(),
                              ws.low_b.as<float>(), ws.dec540.as<float>(), ws.refined.as<float>(), ws.meta.as<float>(), s,
                              &launches, mark,
                              c.mode == Mode::Calibrate ? reinterpret_cast<float*>(stats_.as<double>() + 448) : nullptr,
                              c.mode == Mode::Calibrate ? stats_.as<double>() : nullptr);
    }
    if (c.mode == Mode::Calibrate) {
        // activation maxima only
    } else if (predict) {
        // one region per frame, covering it: metadata NHWC [h/2, w/2, 64] per frame
        const size_t bytes = 4 * packed * 64;
        const char* meta = tcr ? ws.raw.as<char>() : ws.meta.as<char>();
        for (int i = 0; i < R; ++i) {
            const int f = grp.regions[first + i].frame;
            char* out = static_cast<char*>(c.host ? dst_.get() : c.dst) + size_t(f) * bytes;
            AEISU_CUDA(cudaMemcpyAsync(out, meta + size_t(i) * bytes, bytes, cudaMemcpyDeviceToDevice, s));
        }
    } else if (tcr) {
        if (!fuse)
            launch_tc_head(src, rs, dst, ws.meta.get(), head_img_, flag_.as<int>(), flag_.as<int>() + 1, s, &launches);
    } else {
        launch_f32_head(src, rs, dst, ws.meta.as<float>(), base_, basis_, flag_.as<int>(), s, &launches);
    }
    record(5, s);
    launches_ += uint64_t(launches);
}

// Host-buffer upscale of several frames from and to page-locked memory: frames go through in
// chunks, so the upload of chunk i+1 and the download of chunk i-1 (two copy streams) overlap
// the kernels of chunk i on the compute stream.  Frames are independent, so a chunk is a
// complete upscale call of its own; the device buffers hold the whole batch, so no chunk waits
// for a buffer slot.
void Engine::run_pipelined(const Call& c, cudaStream_t s) {
    const int chunks = std::min(c.n, 16);
    const int per = (c.n + chunks - 1) / chunks;
    const size_t in_frame = size_t(3) * c.h * c.w, out_frame = size_t(12) * c.h * c.w;
    src_.ensure(in_frame * c.n, s);
    dst_.ensure(out_frame * c.n, s);
    while (chunk_ev_.size() < size_t(2 * chunks + 1)) {
        cudaEvent_t e;
        AEISU_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        chunk_ev_.push_back(e);
    }
    // the copy streams start after everything already queued on the compute stream
    AEISU_CUDA(cudaStreamWaitEvent(copy_in_, ev_[0], 0));
    AEISU_CUDA(cudaStreamWaitEvent(copy_out_, ev_[0], 0));
    AEISU_CUDA(cudaMemsetAsync(flag_.get(), 0, 2 * sizeof(int), s));  // [0] non-finite, [1] pipeline error
    const uint8_t* hsrc = static_cast<const uint8_t*>(c.src);
    uint8_t* hdst = static_cast<uint8_t*>(c.dst);
    for (int i = 0, f0 = 0; f0 < c.n; ++i, f0 += per) {
        const int k = std::min(per, c.n - f0);
        cudaEvent_t uploaded = chunk_ev_[2 * i], computed = chunk_ev_[2 * i + 1];
        uint8_t* dsrc = src_.as<uint8_t>() + in_frame * f0;
        uint8_t* ddst = dst_.as<uint8_t>() + out_frame * f0;
        AEISU_CUDA(cudaMemcpyAsync(dsrc, hsrc + in_frame * f0, in_frame * k, cudaMemcpyHostToDevice, copy_in_));
        AEISU_CUDA(cudaEventRecord(uploaded, copy_in_));
        AEISU_CUDA(cudaStreamWaitEvent(s, uploaded, 0));
        record(0, s);
        Call part = c;
        part.n = k;
        const Geometry& g = plan(part);
        SrcDesc src{dsrc, 0, c.h, c.w, g.pad_y, g.pad_x};
        DstDesc dst{ddst, 0, 2 * g.out_h, 2 * g.out_w, g.pad_y, g.pad_x};
        for (const auto& grp : g.groups) run_group(part, g, grp, src, dst, s);
        AEISU_CUDA(cudaEventRecord(computed, s));
        AEISU_CUDA(cudaStreamWaitEvent(copy_out_, computed, 0));
        AEISU_CUDA(cudaMemcpyAsync(hdst + out_frame * f0, ddst, out_frame * k, cudaMemcpyDeviceToHost, copy_out_));
    }
    // the call ends on the compute stream once the last download has landed
    AEISU_CUDA(cudaEventRecord(chunk_ev_[2 * chunks], copy_out_));
    AEISU_CUDA(cudaStreamWaitEvent(s, chunk_ev_[2 * chunks], 0));
    AEISU_CUDA(cudaEventRecord(ev_[6], s));
    finish_host_call(c, s, false, 0);
}

void Engine::finish_host_call(const Call& c, cudaStream_t s, bool staged, size_t dst_bytes) {
    wait(s, timeout_ms_);
    if (staged) std::memcpy(c.dst, staging_.get(), dst_bytes);
    int flag[2] = {0, 0};
    AEISU_CUDA(cudaMemcpy(flag, flag_.get(), sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag[1]) fail(AEISU_ERR_CUDA, "tensor-core pipeline wait expired inside a kernel (code " +
                                          std::to_string(flag[1]) + ")");
    if (flag[0] && c.mode == Mode::Upscale) fail(AEISU_ERR_NONFINITE, "Non-finite model reconstruction");
}

const Geometry& Engine::plan(const Call& c) {
    const std::array<int, 7> key{int(c.mode), c.n, c.h, c.w, c.tile, c.band, c.bands};
    auto it = plan_cache_.find(key);
    if (it != plan_cache_.end()) return it->second;
    Geometry g = c.bands > 0                ? plan_band(c.h, c.w, c.band, c.bands)
                 : (c.mode == Mode::Upscale || c.mode == Mode::Calibrate) ? plan_upscale(c.n, c.h, c.w, c.tile)
                                             : plan_whole(c.n, c.h, c.w);
    if (plan_cache_.size() >= 256) plan_cache_.clear();
    return plan_cache_.emplace(key, std::move(g)).first->second;
}

// Calibration for the SPYR8 exporter: the FP32 controller on the padded frames, exactly as an
// upscale with tile 0 runs it, with running maxima and channel sums.
void Engine::activation_stats(const uint8_t* src, bool host, int n, int h, int w, float* peaks, float* means,
                              cudaStream_t stream) {
    DeviceGuard guard(device_);
    require(src != nullptr && peaks != nullptr, "source and peaks must not be null");
    if (precision_ != AEISU_PRECISION_FP32)
        fail(AEISU_ERR_UNSUPPORTED, "activation statistics are measured on the FP32 route (open the folded checkpoint with precision fp32)");
    Call c{Mode::Calibrate, src, 0, nullptr, 0, n, h, w, 0, host, stream};
    const Geometry& g = plan(c);
    cudaStream_t s = stream ? stream : stream_;
    marks_.clear();
    timings_pending_ = true;
    AEISU_CUDA(cudaEventRecord(ev_[0], s));
    const void* src_ptr = src;
    if (host) {
        const size_t bytes = size_t(n) * 3 * h * w;
        src_.ensure(bytes, s);
        AEISU_CUDA(cudaMemcpyAsync(src_.get(), src, bytes, cudaMemcpyHostToDevice, s));
        src_ptr = src_.get();
    }
    constexpr size_t kStatBytes = 448 * sizeof(double) + 16 * sizeof(float);
    stats_.ensure(kStatBytes, s);
    AEISU_CUDA(cudaMemsetAsync(stats_.get(), 0, kStatBytes, s));
    AEISU_CUDA(cudaMemsetAsync(flag_.get(), 0, 2 * sizeof(int), s));
    record(0, s);
    SrcDesc sd{src_ptr, 0, h, w, g.pad_y, g.pad_x};
    DstDesc dd{nullptr, 0, 2 * g.out_h, 2 * g.out_w, g.pad_y, g.pad_x};
    double packed = 0, low = 0;   // pixels at half and quarter resolution over all regions
    for (const auto& grp : g.groups) {
        run_group(c, g, grp, sd, dd, s);
        packed += double(grp.regions.size()) * (grp.rh / 2) * (grp.rw / 2);
        low += double(grp.regions.size()) * (grp.rh / 4) * (grp.rw / 4);
    }
    char* staged = static_cast<char*>(staging_.ensure(kStatBytes, s));
    AEISU_CUDA(cudaMemcpyAsync(staged, stats_.get(), kStatBytes, cudaMemcpyDeviceToHost, s));
    AEISU_CUDA(cudaEventRecord(ev_[6], s));
    wait(s, timeout_ms_);
    const double* sums = reinterpret_cast<const double*>(staged);
    std::memcpy(peaks, staged + 448 * sizeof(double), 10 * sizeof(float));
    if (means)
        for (int i = 0; i < 448; ++i) means[i] = float(sums[i] / (i < 128 ? packed / 4 : low));
}

void Engine::run(const Call& c) {
    DeviceGuard guard(device_);
    require(c.src != nullptr && c.dst != nullptr, "source and destination must not be null");
    const Geometry& g = plan(c);
    cudaStream_t s = c.stream ? c.stream : stream_;
    if (c.bands == 0 && c.host && c.mode == Mode::Upscale && c.src_kind == 0 && c.dst_kind == 0 && c.n >= 2 &&
        is_pinned(c.src) && is_pinned(c.dst)) {
        marks_.clear();
        timings_pending_ = true;
        AEISU_CUDA(cudaEventRecord(ev_[0], s));
        run_pipelined(c, s);
        return;
    }
    const size_t src_elem = c.src_kind == 0 ? 1 : 4;
    const size_t src_bytes = size_t(c.n) * 3 * c.h * c.w * src_elem;
    size_t dst_bytes;
    if (c.mode == Mode::Predict) dst_bytes = size_t(c.n) * (c.h / 2) * (c.w / 2) * 64 * 4;
    else dst_bytes = size_t(c.n) * 3 * (2 * size_t(g.out_h)) * (2 * size_t(g.out_w)) * (c.dst_kind == 0 ? 1 : 4);

    marks_.clear();
    timings_pending_ = true;
    AEISU_CUDA(cudaEventRecord(ev_[0], s));
    const void* src_ptr = c.src;
    void* dst_ptr = c.dst;
    // byte ranges of the host buffers a call reads and writes: whole buffers, or for a row
    // band the source rows its crop can touch and the output rows of its core
    size_t src_off = 0, src_len = src_bytes, dst_off = 0, dst_len = dst_bytes;
    if (c.bands > 0) {
        src_len = dst_len = 0;
        if (!g.groups.empty()) {
            const Region& r = g.groups[0].regions[0];
            const int rh = g.groups[0].rh;
            const int r0 = std::clamp(r.oy - g.pad_y, 0, c.h - 1), r1 = std::clamp(r.oy + rh - 1 - g.pad_y, 0, c.h - 1);
            const size_t src_row = size_t(3) * c.w * src_elem, dst_row = size_t(6) * c.w * (c.dst_kind == 0 ? 1 : 4);
            src_off = src_row * r0;
            src_len = src_row * (r1 - r0 + 1);
            dst_off = dst_row * 2 * (r.oy + r.cy0 - g.pad_y);
            dst_len = dst_row * 2 * (r.cy1 - r.cy0);
            require(c.src_kind == 0, "row bands take uint8 frames");
        }
    }
    if (c.host) {
        src_.ensure(src_bytes, s);
        dst_.ensure(dst_bytes, s);
        if (src_len)
            AEISU_CUDA(cudaMemcpyAsync(src_.as<char>() + src_off, static_cast<const char*>(c.src) + src_off, src_len,
                                       cudaMemcpyHostToDevice, s));
        src_ptr = src_.get();
        dst_ptr = dst_.get();
    }
    AEISU_CUDA(cudaMemsetAsync(flag_.get(), 0, 2 * sizeof(int), s));  // [0] non-finite, [1] pipeline error
    record(0, s);
    SrcDesc src{src_ptr, c.src_kind, c.h, c.w, g.pad_y, g.pad_x};
    DstDesc dst{dst_ptr, c.dst_kind, 2 * g.out_h, 2 * g.out_w, g.pad_y, g.pad_x};
    for (const auto& grp : g.groups) run_group(c, g, grp, src, dst, s);
    // Pageable destinations go through page-locked staging: a direct copy into pageable
    // memory would block the host without the completion bound.
    const bool staged = c.host && !is_pinned(c.dst);
    if (c.host && dst_len) {
        char* out = staged ? static_cast<char*>(staging_.ensure(dst_len, s)) : static_cast<char*>(c.dst) + dst_off;
        AEISU_CUDA(cudaMemcpyAsync(out, dst_.as<char>() + dst_off, dst_len, cudaMemcpyDeviceToHost, s));
    }
    AEISU_CUDA(cudaEventRecord(ev_[6], s));
    if (c.host) {
        wait(s, timeout_ms_);
        if (staged && dst_len) std::memcpy(static_cast<char*>(c.dst) + dst_off, staging_.get(), dst_len);
        finish_host_call(c, s, false, 0);
    }
}

}  // namespace aeisu
