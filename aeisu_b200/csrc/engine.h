// Per-device execution engine: weights resident on one GPU, workspace, stream, and the
// orchestration of one inference call (padding geometry, tiling into regions, kernel
// launches, host<->device copies, bounded completion wait).
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "kernels.h"
#include "model.h"

namespace aeisu {

class DevBuf {
public:
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf();
    // Grow to at least `bytes`; waits for `s` before releasing an old allocation.
    void* ensure(size_t bytes, cudaStream_t s);
    void reset();
    void* get() const { return p_; }
    size_t capacity() const { return cap_; }
    template <typename T> T* as() const { return static_cast<T*>(p_); }

private:
    void* p_ = nullptr;
    size_t cap_ = 0;
};

// Page-locked host staging buffer (device->host results land here when the caller's
// buffer is pageable, so the completion wait stays bounded).
class HostBuf {
public:
    HostBuf() = default;
    HostBuf(const HostBuf&) = delete;
    HostBuf& operator=(const HostBuf&) = delete;
    ~HostBuf() { reset(); }
    void* ensure(size_t bytes, cudaStream_t s);
    void reset();
    void* get() const { return p_; }

private:
    void* p_ = nullptr;
    size_t cap_ = 0;
};

// One region of the padded grid (a whole frame for tile=0, a crop for tile>0).
struct Region { int frame, oy, ox, cy0, cx0, cy1, cx1; };

struct Geometry {
    int n, h, w;            // input frames and size
    int pad_y, pad_x;       // replicate padding before the top/left edge
    int ph, pw;             // padded grid size
    int out_h, out_w;       // LR extent written to the output (h, w)
    // regions grouped by shape: every group launches as one batch
    struct Group { int rh, rw; std::vector<Region> regions; };
    std::vector<Group> groups;
};

// Padding and tiling of aeisu/runtime.py:70-99.  tile == 0: one region per frame.
Geometry plan_upscale(int n, int h, int w, int tile);
// One region per frame covering an already padded image (FoldedAEISU.forward semantics).
Geometry plan_whole(int n, int h, int w);
// Row band `band` of `bands` of one frame: the padded grid's rows split into equal bands of a
// multiple of 32 rows; the band's crop adds 32 rows above and below (clipped), like the tile
// halos of runtime.py:92-99, over the full padded width.  Its core pixels equal the
// whole-frame result (the controller's receptive field is smaller than the halo).
Geometry plan_band(int h, int w, int band, int bands);

enum class Mode { Upscale, Forward, Predict, Calibrate };

struct Call {
    Mode mode;
    const void* src; int src_kind;  // 0 u8 HWC, 1 f32 CHW
    void* dst; int dst_kind;        // 0 u8 HWC, 1 f32 CHW (Predict: f32 NHWC metadata)
    int n, h, w, tile;
    bool host;
    cudaStream_t stream;
    int band = 0, bands = 0;        // bands > 0: one row band of a single frame (plan_band)
};

// Device copies of one model's weights.  Sibling engines (aeisu_open_sibling) share one copy;
// it is released with the last of them.
struct ResidentWeights {
    DevBuf w_f32;                // all FP32 tensors, packed
    DevBuf tc_bytes, tc_floats;  // tensor-core routes: operand images, epilogue vectors
};

class Engine {
public:
    Engine(HostModel model, int precision, int device);
    // A sibling of `parent`: same model, precision and device, sharing its device weights, with
    // its own stream, workspace, status flags and timings (SrcPyrCudaRuntime.cu:5392-5402 shares
    // the engine; here only the weights are shared, so siblings may run concurrently).
    struct Sibling {};
    Engine(const Engine& parent, Sibling);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    void run(const Call& call);
    void synchronize(cudaStream_t s, double timeout_ms);
    // FP32 route over n uint8 frames (tile 0, no reconstruction), returning (host) in peaks[10]
    // the max |x| of each activation the mixed route quantises and, if means is not null, in
    // means[448] the mean of every input channel of the FP8 layers; waits for completion.
    void activation_stats(const uint8_t* src, bool host, int n, int h, int w, float* peaks, float* means,
                          cudaStream_t stream);

    const std::string& report() const { return report_; }
    uint64_t device_bytes() const;
    uint64_t launches() const { return launches_; }
    // Stage times of the last call (waits for it to finish when stage marks are pending).
    const aeisu_timings& timings();
    void set_detailed(bool on) { detailed_ = on; }
    // Tensor-core upscales reconstruct in a separate head kernel over coefficients kept in HBM
    // (default, the faster) or inside the controller's last kernel (same output bit for bit).
    void set_fused_head(bool on) { fused_head_ = on; }
    void set_timeout(double ms) { timeout_ms_ = ms; }
    void set_workspace_cap(size_t bytes) { workspace_cap_ = bytes; }
    int precision() const { return precision_; }
    int device() const { return device_; }

    // Device-resident weights and status flags, for entry points that run the kernels on
    // buffers they do not take from this engine's workspace.
    struct Resident {
        const TcWeights* tc;
        const uint8_t* head_img;
        const float* stencil;
        const F32Layer* f32;
        const float* base;
        const float* basis;
        int* flags;             // [0] non-finite output, [1] kernel pipeline error
        cudaStream_t stream;
    };
    Resident resident() const {
        return {&tcw_, head_img_, stencil_, f32_layers_, base_, basis_,
                flag_.as<int>(), stream_};
    }
    void count_launches(int n) { launches_ += uint64_t(n); }

private:
    struct DeviceGuard;
    void upload_weights();
    void create_streams();
    // Intermediate activations of one batch of regions.  Large batches run as two halves on two
    // streams at once (the compute stream and lane_), each with its own workspace: the two
    // halves' kernels fill each other's tails and waits.
    struct Workspace {
        DevBuf enc540, low_a, low_b, dec540, refined, meta, encu, raw;
    };
    void run_group(const Call& c, const Geometry& g, const Geometry::Group& grp, const SrcDesc& src,
                   const DstDesc& dst, cudaStream_t s);
    void run_regions(const Call& c, const Geometry::Group& grp, size_t first, int R, const SrcDesc& src,
                     const DstDesc& dst, cudaStream_t s, Workspace& ws);
    void run_pipelined(const Call& c, cudaStream_t s);
    void finish_host_call(const Call& c, cudaStream_t s, bool staged, size_t dst_bytes);
    void wait(cudaStream_t s, double timeout_ms);
    void record(int stage, cudaStream_t s);
    bool fused(const Call& c) const {
        return fused_head_ && precision_ != AEISU_PRECISION_FP32 && (c.mode == Mode::Upscale || c.mode == Mode::Forward);
    }

    HostModel model_;
    int precision_, device_;
    cudaStream_t stream_ = nullptr;
    cudaStream_t copy_in_ = nullptr, copy_out_ = nullptr;   // host<->device copies of pipelined calls
    std::string report_;
    double timeout_ms_ = 60000.0;
    bool detailed_ = false;
    bool fused_head_ = false;
    uint64_t launches_ = 0;
    aeisu_timings timings_{};

    // resident weights (shared with siblings) and the pointers into them
    DevBuf stats_;               // calibration: channel sums (double[448]) then maxima (float[10])
    std::shared_ptr<ResidentWeights> weights_;
    const float* stencil_ = nullptr;
    const float* base_ = nullptr;
    const float* basis_ = nullptr;
    F32Layer f32_layers_[kLayerCount]{};
    TcWeights tcw_{};
    const uint8_t* head_img_ = nullptr;

    // planned geometry per call shape (mode, n, h, w, tile, band, bands)
    std::map<std::array<int, 7>, Geometry> plan_cache_;
    const Geometry& plan(const Call& c);
    // region tables per call geometry (mode, n, h, w, tile, group shape, first region, regions,
    // band, bands)
    using TableKey = std::array<int, 10>;
    std::map<TableKey, std::unique_ptr<DevBuf>> table_cache_;

    // workspace
    DevBuf src_, dst_, tables_, flag_;
    HostBuf staging_;
    Workspace ws_[2];
    cudaStream_t lane_ = nullptr;                     // second stream of a split batch
    cudaEvent_t fork_ = nullptr, join_ = nullptr;
    size_t workspace_cap_ = size_t(6) << 30;

    // timing events: [0] call start, [1]/[2] detailed stage marks, [6] call end, [7] waits
    cudaEvent_t ev_[8] = {};
    std::vector<cudaEvent_t> pool_;                // stage-mark events, reused across calls
    std::vector<cudaEvent_t> chunk_ev_;            // pipelined calls: 2 events per frame chunk
    std::vector<std::pair<int, int>> marks_;       // (stage closed by this mark, pool index)
    bool timings_pending_ = false;
};

}  // namespace aeisu
