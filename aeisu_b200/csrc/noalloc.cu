// aeisu_upscale_u8_noalloc: the device-I/O uint8 upscale, run entirely inside a fixed,
// statically sized device array instead of the handle's growable workspace.
//
// Some host programs cannot call cudaMalloc at the point where they need a frame upscaled:
// code running inside a real-time presentation loop that must not block on the allocator
// (cudaMalloc can synchronise the device), processes whose memory budget is fixed at start-up
// by another component, or hosts that hand the library raw device pointers from a pool they
// manage themselves.  For them this entry point allocates nothing, anywhere: the controller's
// intermediate activations, the region table and the coefficient buffer all live in
// `g_noalloc_scratch` below.  The caller still provides the input and output device buffers,
// and the handle (opened earlier, when allocation was allowed) provides the weights.
//
// Limits and sharing:
//  * The array holds kNoAllocScratchBytes (64 MiB) on every GPU that loads this library, for
//    the life of the process.  A frame needs about 80 bytes of scratch per padded input pixel
//    on the mixed route, 96 on FP16 and INT8 and 224 on FP32 (the sums of the buffer sizes in
//    upscale_u8_noalloc), so frames above about 0.83, 0.69 and 0.29 Mpixel of padded input are
//    rejected with AEISU_ERR_INVALID_ARG (960x540 fits the tensor-core routes, 640x360 FP32).
//    Batches run in as many passes of whole frames as the array needs.
//  * The array is shared by every call on a device and keeps the last call's contents.
//    Nothing in it has to start at zero (every byte a kernel reads was written earlier in the
//    same call), but two calls whose GPU work overlaps in time -- on different streams, or
//    from different handles on one device -- race on it.  Serialise them.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current), and the first launch of each kernel on
//    a device may set its shared-memory attribute and add entries to the host-side caches of
//    those attributes and of the TMA tensor maps over the array (one per shape); make that
//    first call before capturing a CUDA graph on the stream.  No
//    device memory is ever allocated.  The address is cached for the life of the process:
//    after cudaDeviceReset it is stale, so the library must not outlive a reset of the device.
#include <cuda_runtime.h>

#include <mutex>

#include "common.h"
#include "engine.h"
#include "kernels.h"
#include "noalloc.h"

namespace aeisu {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;
constexpr size_t kTableBytes = 64 * 1024;   // region table at the front of the array

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
void* scratch_for(int device) {
    require(device >= 0 && device < kMaxDevices, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            fail(AEISU_ERR_CUDA, std::string("cudaGetSymbolAddress of the no-allocation scratch failed: ") +
                                     cudaGetErrorString(e));
        g_scratch_addr[device] = p;
    }
    return g_scratch_addr[device];
}

// Region table of `count` whole frames starting at `first`: origin (0, 0) on the padded grid,
// core = the unpadded frame (runtime.py:81-84, tile = 0).
__global__ void k_fill_regions(int4* table, int count, int first, int pad_y, int pad_x, int h, int w) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    table[i] = make_int4(first + i, 0, 0, 0);
    table[count + i] = make_int4(pad_y, pad_x, pad_y + h, pad_x + w);
}

struct ScopedDevice {
    int prev = -1;
    explicit ScopedDevice(int dev) {
        AEISU_CUDA(cudaGetDevice(&prev));
        if (prev != dev) AEISU_CUDA(cudaSetDevice(dev));
    }
    ~ScopedDevice() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
    }
};

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

void upscale_u8_noalloc(Engine& e, const uint8_t* src, int n, int h, int w, uint8_t* dst, cudaStream_t stream) {
    require(src != nullptr && dst != nullptr, "source and destination must be device pointers");
    require(n >= 1 && h >= 1 && w >= 1, "Expected CHW RGB image");
    ScopedDevice guard(e.device());
    uint8_t* scratch = static_cast<uint8_t*>(scratch_for(e.device()));
    const Engine::Resident res = e.resident();
    cudaStream_t s = stream ? stream : res.stream;
    // padded grid of runtime.py:79-84
    const int ey = (32 - h % 32) % 32, ex = (32 - w % 32) % 32;
    const int pad_y = 16 + ey / 2, pad_x = 16 + ex / 2, ph = h + 32 + ey, pw = w + 32 + ex;
    const size_t packed = size_t(ph / 2) * (pw / 2), low = size_t(ph / 4) * (pw / 4);
    const int prec = e.precision();
    const bool tcr = prec != AEISU_PRECISION_FP32, fp8 = prec == AEISU_PRECISION_MIXED;
    // per-frame scratch, laid out as the engine's workspace for the same precision
    const size_t enc_b = align256(tcr ? packed * 64 : packed * 32 * 4);
    const size_t encu_b = align256(tcr ? low * (fp8 ? 128 : 256) : 0);
    const size_t low_b = align256(tcr ? low * (fp8 ? 64 : 128) : low * 64 * 4);
    const size_t dec_b = align256(tcr ? packed * 64 : packed * 32 * 4);
    const size_t ref_b = align256(tcr ? 0 : packed * 64 * 4);
    const size_t meta_b = align256(tcr ? size_t(ph) * pw * 32 : packed * 64 * 4);
    const size_t per_frame = enc_b + encu_b + 2 * low_b + dec_b + ref_b + meta_b;
    const size_t room = kNoAllocScratchBytes - kTableBytes;
    if (per_frame > room)
        fail(AEISU_ERR_INVALID_ARG,
             "frame " + std::to_string(w) + "x" + std::to_string(h) + " needs " + std::to_string(per_frame) +
                 " bytes of scratch; the no-allocation entry point has " + std::to_string(room));
    const int chunk = int(std::min<size_t>(room / per_frame, kTableBytes / (2 * sizeof(int4))));
    SrcDesc sd{src, 0, h, w, pad_y, pad_x};
    DstDesc dd{dst, 0, 2 * h, 2 * w, pad_y, pad_x};
    AEISU_CUDA(cudaMemsetAsync(res.flags, 0, 2 * sizeof(int), s));
    int launches = 0;
    for (int first = 0; first < n; first += chunk) {
        const int R = std::min(chunk, n - first);
        int4* table = reinterpret_cast<int4*>(scratch);
        k_fill_regions<<<(R + 127) / 128, 128, 0, s>>>(table, R, first, pad_y, pad_x, h, w);
        ++launches;
        RegionSet rs{};
        rs.regions = table;
        rs.cores = table + R;
        rs.R = R; rs.rh = ph; rs.rw = pw; rs.core_h = h; rs.core_w = w;
        uint8_t* p = scratch + kTableBytes;
        uint8_t* enc540 = p; p += enc_b * R;
        uint8_t* encu = p; p += encu_b * R;
        uint8_t* low_a = p; p += low_b * R;
        uint8_t* low_b_ = p; p += low_b * R;
        uint8_t* dec540 = p; p += dec_b * R;
        uint8_t* refined = p; p += ref_b * R;
        uint8_t* meta = p;
        StageMark none;
        if (tcr) {
            launch_tc_controller(tc_route_of(prec), sd, rs, *res.tc, enc540, encu, low_a, low_b_, dec540, meta, nullptr,
                                 res.flags + 1, s, &launches, none);
            launch_tc_head(sd, rs, dd, meta, res.head_img, res.flags, res.flags + 1, s, &launches);
        } else {
            launch_f32_controller(sd, rs, res.stencil, res.f32, reinterpret_cast<float*>(enc540),
                                  reinterpret_cast<float*>(low_a), reinterpret_cast<float*>(low_b_),
                                  reinterpret_cast<float*>(dec540), reinterpret_cast<float*>(refined),
                                  reinterpret_cast<float*>(meta), s, &launches, none);
            launch_f32_head(sd, rs, dd, reinterpret_cast<float*>(meta), res.base, res.basis, res.flags, s, &launches);
        }
    }
    AEISU_CUDA(cudaGetLastError());
    e.count_launches(launches);
}

}  // namespace aeisu
