#include "tmap.h"

#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "common.h"

namespace aeisu {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) fail(AEISU_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

}  // namespace

CUtensorMap make_row_window_map(const void* base, int R, int H, int nch, int W, int win, int box_ch) {
    if (box_ch == 0) box_ch = nch;
    require(win >= 1 && win <= 128 && nch >= 1 && nch <= 256 && box_ch >= 1 && box_ch <= nch,
            "tensor map box out of range");
    require((reinterpret_cast<uintptr_t>(base) & 15) == 0, "tensor map base must be 16-byte aligned");
    // A map depends only on its arguments, and calls reuse the same workspace: encode each once.
    using Key = std::tuple<const void*, int, int, int, int, int, int>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{base, R, H, nch, W, win, box_ch};
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    CUtensorMap map{};
    // 8-byte elements, two per pixel: a row window is one box row of 2*win elements per chunk
    // (up to 2 KB contiguous), which TMA moves in wide requests.
    const cuuint64_t dims[4] = {2 * cuuint64_t(W), cuuint64_t(nch), cuuint64_t(H), cuuint64_t(R)};
    const cuuint64_t strides[3] = {cuuint64_t(W) * 16, cuuint64_t(nch) * W * 16, cuuint64_t(H) * nch * W * 16};
    const cuuint32_t box[4] = {2 * cuuint32_t(win), cuuint32_t(box_ch), 1, 1};
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<void*>(base), dims, strides,
                                   box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(AEISU_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
    std::lock_guard<std::mutex> lock(mu);
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, map);
    return map;
}

}  // namespace aeisu
