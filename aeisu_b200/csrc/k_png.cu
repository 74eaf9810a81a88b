// PNG encoding on the GPU: the file save_rgb writes (aeisu/runtime.py:23-27: clamp,
// floor(x * 255 + 0.5), 8-bit RGB PNG through PIL), produced from frames already in HBM.
// The decoded pixels are the reference's; the compressed bytes differ (PIL runs zlib at level 6
// with hash chains and lazy matching, this encoder one candidate per position and a greedy
// parse).
//
// Pipeline per call (all frames of the batch at once):
//   k_png_filter   one CTA per image row: the row and the row above are staged in shared
//                  memory, the five PNG filters (None, Sub, Up, Average, Paeth) are scored by
//                  the sum of |residual| as signed bytes (the usual adaptive choice) and the
//                  filter byte + filtered row are written to the frame's zlib input stream.
//   k_png_deflate  one CTA per 60 KiB segment of that stream: LZ77 match candidates from a
//                  shared-memory hash table, a greedy parse per thread, the segment's Huffman
//                  codes (deflate.cuh, one thread; a literal-only code is built beside it by
//                  another thread and the smaller block wins), a block scan of the per-thread
//                  bit counts, then every thread packs its tokens into a shared-memory bit
//                  buffer.  A segment is one dynamic block; all but the last end with an empty
//                  stored block so that the next starts on a byte boundary.  A segment whose
//                  code would not be smaller than the raw bytes is stored.  Adler-32 partial
//                  sums of the segment come out of the hashing pass.
//   k_png_layout   one CTA per frame: segment offsets (scan), Adler-32, the PNG framing.
//   k_png_gather   copies every segment to its place in the file.
//   k_png_crc      CRC-32 of the IDAT chunk: 256 bytes per thread (table), combined across
//                  a warp and a CTA by multiplying with x^(8 * length) mod P, the
//                  CRC polynomial (the register after `length` zero bytes), per 128 KiB block.
//   k_png_crc_final combines the blocks the same way and writes the chunk's CRC.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "deflate.cuh"
#include "kernels.h"

namespace aeisu {
namespace {

constexpr int kSeg = 61440;                 // zlib input bytes per deflate segment
constexpr int kSlot = kSeg + 64;            // bytes reserved per coded segment
constexpr int kFiltThreads = 256;
constexpr int kDefThreads = 512;
constexpr int kDefWarps = kDefThreads / 32;
constexpr int kChunk = kSeg / kDefThreads;    // bytes parsed per thread (120)
constexpr int kHashBits = 13;
constexpr int kDefSmem = kSlot + 2 * kSeg;    // bit buffer (hash table before it) + candidates
constexpr int kCrcChunk = 256;              // bytes per thread
constexpr int kCrcThreads = 512;
constexpr long long kCrcSpan = (long long)kCrcChunk * kCrcThreads;
constexpr uint32_t kPoly = 0xEDB88320u;     // CRC-32 (ISO-HDLC), bit-reflected
constexpr int kPrefix = 43;                 // signature, IHDR, IDAT length + type, zlib header
constexpr int kSuffix = 20;                 // Adler-32, IDAT CRC, IEND
constexpr int kIdatType = 37;               // offset of "IDAT" (the CRC covers type + data)
constexpr int kMaxWidth = 32768;

struct PngGeom {
    int n, h, w, nseg;
    long long row;      // 3w + 1 bytes per filtered row
    long long U;        // zlib input bytes per frame
    long long ustride;  // frame stride of the zlib input (16-byte multiple)
    long long fstride;  // frame stride of the assembled files
    int crc_blocks;     // CRC blocks launched per frame (enough for the largest file)
};

struct CrcTables {
    uint32_t byte_pow[40];   // x^(8 * 2^j) mod P
    uint32_t block_pow[32];  // x^(8 * kCrcSpan * 2^j) mod P
    uint32_t lane[5];        // x^(8 * kCrcChunk * 2^k) mod P: the warp tree's shifts
    uint32_t warp;           // x^(8 * 32 * kCrcChunk) mod P
};

// Product of two polynomials mod P in the reflected representation (bit 31 = x^0).
__host__ __device__ inline uint32_t gf_mul(uint32_t a, uint32_t b) {
    uint32_t p = 0;
    for (int i = 0; i < 32; ++i) {
        if (a & (0x80000000u >> i)) p ^= b;
        b = (b >> 1) ^ ((b & 1u) ? kPoly : 0u);
    }
    return p;
}

// x^(e * unit) mod P from the table pow[j] = x^(unit * 2^j) mod P.
__host__ __device__ inline uint32_t gf_pow(unsigned long long e, const uint32_t* pow) {
    uint32_t r = 0x80000000u;   // x^0
    for (int j = 0; e; ++j, e >>= 1)
        if (e & 1ull) r = gf_mul(r, pow[j]);
    return r;
}

__device__ __forceinline__ uint8_t quantize(float v) {
    // save_rgb: clamp(0, 1), floor(x * 255 + 0.5) in float32, then uint8
    const float c = fminf(fmaxf(v, 0.f), 1.f);
    return uint8_t(floorf(__fadd_rn(__fmul_rn(c, 255.f), 0.5f)));
}

__device__ __forceinline__ int paeth(int a, int b, int c) {
    const int p = a + b - c, pa = abs(p - a), pb = abs(p - b), pc = abs(p - c);
    return (pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c);
}

__device__ __forceinline__ uint8_t filtered(int type, int x, int a, int b, int c) {
    switch (type) {
        case 1: return uint8_t(x - a);
        case 2: return uint8_t(x - b);
        case 3: return uint8_t(x - ((a + b) >> 1));
        case 4: return uint8_t(x - paeth(a, b, c));
        default: return uint8_t(x);
    }
}

// kind 0: uint8 HWC frames; kind 1: float32 CHW frames quantised as save_rgb does.
__global__ void __launch_bounds__(kFiltThreads) k_png_filter(const void* __restrict__ src, int kind, PngGeom g,
                                                             uint8_t* __restrict__ filt) {
    extern __shared__ uint8_t srow[];
    const int y = blockIdx.x, f = blockIdx.y, t = threadIdx.x;
    const int R = 3 * g.w;
    uint8_t* cur = srow;
    uint8_t* prev = srow + R;
    for (int k = 0; k < 2; ++k) {
        const int yy = y - k;
        uint8_t* dst = k ? prev : cur;
        for (int i = t; i < R; i += kFiltThreads) {
            uint8_t v = 0;
            if (yy >= 0) {
                if (kind == 0) {
                    v = static_cast<const uint8_t*>(src)[(size_t(f) * g.h + yy) * R + i];
                } else {
                    const int x = i / 3, c = i - 3 * x;
                    v = quantize(static_cast<const float*>(src)[((size_t(f) * 3 + c) * g.h + yy) * g.w + x]);
                }
            }
            dst[i] = v;
        }
    }
    __syncthreads();
    unsigned sum[5] = {0, 0, 0, 0, 0};
    for (int i = t; i < R; i += kFiltThreads) {
        const int x = cur[i], a = i >= 3 ? cur[i - 3] : 0, b = prev[i], c = i >= 3 ? prev[i - 3] : 0;
#pragma unroll
        for (int k = 0; k < 5; ++k) sum[k] += abs(int(int8_t(filtered(k, x, a, b, c))));
    }
    __shared__ unsigned s_sum[kFiltThreads / 32][5];
    __shared__ int s_type;
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        unsigned v = sum[k];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
        if ((t & 31) == 0) s_sum[t >> 5][k] = v;
    }
    __syncthreads();
    if (t == 0) {
        unsigned long long best = ~0ull;
        int type = 0;
        for (int k = 0; k < 5; ++k) {
            unsigned long long s = 0;
            for (int w = 0; w < kFiltThreads / 32; ++w) s += s_sum[w][k];
            if (s < best) best = s, type = k;
        }
        s_type = type;
    }
    __syncthreads();
    const int type = s_type;
    uint8_t* out = filt + size_t(f) * g.ustride + size_t(y) * g.row;
    if (t == 0) out[0] = uint8_t(type);
    for (int i = t; i < R; i += kFiltThreads) {
        const int x = cur[i], a = i >= 3 ? cur[i - 3] : 0, b = prev[i], c = i >= 3 ? prev[i - 3] : 0;
        out[1 + i] = filtered(type, x, a, b, c);
    }
}

// Bit writer into a shared-memory word buffer, LSB first; words may be shared with the
// neighbouring writers, so every word is OR-ed in.
struct BitOut {
    uint32_t* buf;
    unsigned long long pos;   // absolute bit position of acc's bit 0
    uint64_t acc = 0;
    int n = 0;
    __device__ void flush32(uint32_t v) {
        const unsigned long long w = pos >> 5;
        const int sh = int(pos & 31);
        atomicOr(&buf[w], v << sh);
        if (sh) atomicOr(&buf[w + 1], v >> (32 - sh));
    }
    __device__ void put(uint32_t v, int bits) {
        acc |= uint64_t(v) << n;
        n += bits;
        if (n >= 32) {
            flush32(uint32_t(acc));
            pos += 32;
            acc >>= 32;
            n -= 32;
        }
    }
    __device__ void finish() {
        if (n) flush32(uint32_t(acc) & (n == 32 ? 0xffffffffu : ((1u << n) - 1u)));
        pos += n;
        n = 0;
        acc = 0;
    }
};

// One CTA per segment.  Phase A finds, for every position, the nearest earlier position with
// the same four bytes (a hash table of last positions in shared memory, filled in rounds of
// kDefThreads positions: a position sees the positions of earlier rounds, reaching back over
// the previous 32 KiB of the frame's stream, so matches may cross into the previous segment).
// Pass 1: each thread parses its 120 bytes greedily (longest of the hash candidate, distance 1
// and the row above, at least 4 bytes, cut at the thread's end), keeps its tokens in global
// scratch and counts symbols.  Thread 0 builds the codes of that parse, thread 32 the codes of
// a literal-only block of the same bytes; the smaller wins (or stored bytes, if smaller still).
// Pass 2 sums each thread's bits for the scan; pass 3 packs them.
__device__ __forceinline__ uint32_t hash4(const uint8_t* p) {
    const uint32_t v = uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24;
    return (v * 2654435761u) >> (32 - kHashBits);
}

__global__ void __launch_bounds__(kDefThreads, 1) k_png_deflate(PngGeom g, const uint8_t* __restrict__ filt,
                                                                uint8_t* __restrict__ slots, uint32_t* __restrict__ tokens,
                                                                uint32_t* seg_bytes, unsigned long long* seg_s1,
                                                                unsigned long long* seg_s2) {
    extern __shared__ __align__(16) uint8_t dsm[];
    uint32_t* obuf = reinterpret_cast<uint32_t*>(dsm);             // kSlot bytes; the hash table before
    int* table = reinterpret_cast<int*>(dsm);                       // (1 << kHashBits) ints
    uint16_t* dist16 = reinterpret_cast<uint16_t*>(dsm + kSlot);    // kSeg: hash candidate distance
    __shared__ uint32_t hist[kDefWarps][defl::kLit];
    __shared__ uint32_t dhist[kDefWarps][defl::kDist];
    __shared__ uint32_t freq[2][defl::kLit];   // [0] parse, [1] literal only
    __shared__ uint32_t dfreq[2][defl::kDist];
    __shared__ uint32_t wt[2][2 * defl::kLit];
    __shared__ uint16_t par[2][2 * defl::kLit], sorted[2][defl::kLit];
    __shared__ defl::Header hd[2];
    __shared__ unsigned long long s_red[2][kDefWarps];
    __shared__ unsigned long long s_scan[kDefWarps];
    __shared__ unsigned long long s_body[2];
    __shared__ int s_m[2];
    const int seg = blockIdx.x, f = blockIdx.y, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const long long fbase = (long long)seg * kSeg;
    const int len = int(std::min<long long>(kSeg, g.U - fbase));
    const bool final = seg == g.nseg - 1;
    const uint8_t* frame = filt + size_t(f) * g.ustride;
    const uint8_t* in = frame + fbase;
    uint8_t* slot = slots + (size_t(f) * g.nseg + seg) * kSlot;
    uint32_t* tok = tokens + (size_t(f) * g.nseg + seg) * kSeg;   // [kChunk][kDefThreads]
    for (int i = t; i < kDefWarps * defl::kLit; i += kDefThreads) (&hist[0][0])[i] = 0;
    for (int i = t; i < kDefWarps * defl::kDist; i += kDefThreads) (&dhist[0][0])[i] = 0;
    for (int i = t; i < (1 << kHashBits); i += kDefThreads) table[i] = -1;
    if (t < 2) s_body[t] = 0;
    __syncthreads();
    // phase A: hash candidates, and the Adler-32 sums s1 = sum b, s2 = sum (len - j) b_j
    unsigned long long s1 = 0, s2 = 0;
    const long long ws = fbase > defl::kWindow ? fbase - defl::kWindow : 0;
    for (long long r0 = ws; r0 < fbase + len; r0 += kDefThreads) {
        const long long p = r0 + t;
        const bool inseg = p >= fbase && p < fbase + len;
        const bool hashed = p < fbase + len && p + 4 <= g.U;
        uint32_t h = 0;
        if (hashed) h = hash4(frame + p);
        if (inseg) {
            int d = 0;
            if (hashed) {
                const int c = table[h];
                if (c >= 0 && p - c <= defl::kWindow) d = int(p - c);
            }
            dist16[p - fbase] = uint16_t(d);   // 32768 fits; 0 = no candidate
            const uint32_t b = frame[p];
            s1 += b;
            s2 += (unsigned long long)(fbase + len - p) * b;
        }
        __syncthreads();
        if (hashed) atomicMax(&table[h], int(p));
        __syncthreads();
    }
    for (int o = 16; o > 0; o >>= 1) {
        s1 += __shfl_down_sync(0xffffffffu, s1, o);
        s2 += __shfl_down_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) s_red[0][warp] = s1, s_red[1][warp] = s2;
    // pass 1: greedy parse of this thread's bytes
    const int i0 = std::min(len, t * kChunk), i1 = std::min(len, i0 + kChunk);
    int ntok = 0;
    for (int i = i0; i < i1;) {
        const long long p = fbase + i;
        const int lim = min(int(defl::kMaxMatch), i1 - i);
        int best = 0, bd = 0;
        const int cand[3] = {int(dist16[i]), 1, int(g.row)};
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int d = cand[k];
            if (d <= 0 || d > defl::kWindow || p < d || lim < defl::kMinMatch) continue;
            const uint8_t* a = frame + p;
            const uint8_t* b = a - d;
            int L = 0;
            while (L < lim && a[L] == b[L]) ++L;
            if (L > best) best = L, bd = d;
        }
        uint32_t tk;
        if (best >= defl::kMinMatch) {
            tk = defl::match_token(best, bd);
            int ne, ev;
            atomicAdd(&hist[warp][defl::length_symbol(best, ne, ev)], 1u);
            atomicAdd(&dhist[warp][defl::distance_symbol(bd, ne, ev)], 1u);
            i += best;
        } else {
            tk = in[i];
            atomicAdd(&hist[warp][tk], 1u);
            ++i;
        }
        tok[size_t(ntok++) * kDefThreads + t] = tk;
    }
    __syncthreads();
    if (t < defl::kLit) {   // parse frequencies; literal-only frequencies = byte counts
        uint32_t c = t == 256 ? 1u : 0u;
        for (int w = 0; w < kDefWarps; ++w) c += hist[w][t];
        freq[0][t] = c;
    }
    if (t < defl::kDist) {
        uint32_t c = 0;
        for (int w = 0; w < kDefWarps; ++w) c += dhist[w][t];
        dfreq[0][t] = c;
        dfreq[1][t] = 0;
    }
    if (t == 0) {
        unsigned long long a = 0, b = 0;
        for (int w = 0; w < kDefWarps; ++w) a += s_red[0][w], b += s_red[1][w];
        seg_s1[size_t(f) * g.nseg + seg] = a;
        seg_s2[size_t(f) * g.nseg + seg] = b;
    }
    // byte histogram for the literal-only alternative (reuses the per-warp tables)
    __syncthreads();
    for (int i = t; i < kDefWarps * defl::kLit; i += kDefThreads) (&hist[0][0])[i] = 0;
    __syncthreads();
    for (int i = i0; i < i1; ++i) atomicAdd(&hist[warp][in[i]], 1u);
    __syncthreads();
    if (t < defl::kLit) {
        uint32_t c = t == 256 ? 1u : 0u;
        for (int w = 0; w < kDefWarps; ++w) c += hist[w][t];
        freq[1][t] = c;
    }
    __syncthreads();
    // used symbols of both alphabets in ascending (frequency, symbol) order, by rank
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        const bool used = t < defl::kLit && freq[a][t] > 0;
        const int m = __syncthreads_count(used);
        if (t == 0) s_m[a] = m;
        if (used) {
            const uint32_t ft = freq[a][t];
            int rank = 0;
            for (int j = 0; j < defl::kLit; ++j) {
                const uint32_t fj = freq[a][j];
                rank += fj > 0 && (fj < ft || (fj == ft && j < t));
            }
            sorted[a][rank] = uint16_t(t);
        }
    }
    __syncthreads();
    if (t == 0 || t == 32) {   // the two codes are built by threads of different warps at once
        const int a = t ? 1 : 0;
        defl::build_header(freq[a], s_m[a], dfreq[a], hd[a], defl::HuffScratch{wt[a], par[a], sorted[a]});
    }
    __syncthreads();
    // body sizes of both alternatives (exact: the parse's tokens, the literal bytes)
    unsigned long long mine[2] = {0, 0};
    for (int k = 0; k < ntok; ++k) mine[0] += defl::token_bits(hd[0], tok[size_t(k) * kDefThreads + t]);
    for (int i = i0; i < i1; ++i) mine[1] += hd[1].lit_len[in[i]];
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        unsigned long long v = mine[a];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
        if (lane == 0) atomicAdd(&s_body[a], v);
    }
    // the hash table is dead: the region becomes the output bit buffer
    for (int i = t; i < kSlot / 4; i += kDefThreads) obuf[i] = 0;
    __syncthreads();
    unsigned long long bytes[2];
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        const unsigned long long bits = hd[a].bits + s_body[a] + hd[a].lit_len[256];
        bytes[a] = final ? (bits + 7) / 8 : (bits + 3 + 7) / 8 + 4;
    }
    const int mode = bytes[1] < bytes[0] ? 1 : 0;
    const unsigned long long huff_bytes = bytes[mode];
    if (huff_bytes >= 5ull + len) {   // stored
        if (t == 0) {
            slot[0] = final ? 1 : 0;   // BFINAL, BTYPE = 00, padding
            slot[1] = uint8_t(len), slot[2] = uint8_t(len >> 8);
            slot[3] = uint8_t(~len), slot[4] = uint8_t((~len) >> 8);
            seg_bytes[size_t(f) * g.nseg + seg] = 5u + len;
        }
        for (int i = t; i < len; i += kDefThreads) slot[5 + i] = in[i];
        return;
    }
    const defl::Header& H = hd[mode];
    unsigned long long incl = mine[mode];
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_scan[warp] = incl;
    if (t == 0) {
        BitOut bo{obuf, 0};
        defl::write_header(H, final, [&](uint32_t v, int b) { bo.put(v, b); });
        bo.finish();
    }
    __syncthreads();
    unsigned long long before = 0;
    for (int w = 0; w < warp; ++w) before += s_scan[w];
    BitOut bo{obuf, (unsigned long long)H.bits + before + incl - mine[mode]};
    if (mode == 0) {
        for (int k = 0; k < ntok; ++k)
            defl::put_token(H, tok[size_t(k) * kDefThreads + t], [&](uint32_t v, int b) { bo.put(v, b); });
    } else {
        for (int i = i0; i < i1; ++i) bo.put(H.lit_code[in[i]], H.lit_len[in[i]]);
    }
    bo.finish();
    if (t == kDefThreads - 1) {   // end of block, then byte alignment
        BitOut e{obuf, bo.pos};
        e.put(H.lit_code[256], H.lit_len[256]);
        if (!final) e.put(0u, 3);   // empty stored block: BFINAL 0, BTYPE 00, then LEN/NLEN
        e.finish();
        if (!final) {
            BitOut z{obuf, (e.pos + 7) / 8 * 8};
            z.put(0u, 16);
            z.put(0xFFFFu, 16);
            z.finish();
        }
        seg_bytes[size_t(f) * g.nseg + seg] = uint32_t(huff_bytes);
    }
    __syncthreads();
    uint32_t* dst = reinterpret_cast<uint32_t*>(slot);
    for (int i = t; i < int((huff_bytes + 3) / 4); i += kDefThreads) dst[i] = obuf[i];
}

__device__ __forceinline__ void put_be32(uint8_t* p, uint32_t v) {
    p[0] = uint8_t(v >> 24), p[1] = uint8_t(v >> 16), p[2] = uint8_t(v >> 8), p[3] = uint8_t(v);
}

struct PngHead {
    uint8_t bytes[kPrefix];   // signature, IHDR chunk, IDAT length (patched), "IDAT", zlib header
};

__global__ void k_png_layout(PngGeom g, PngHead head, const uint32_t* seg_bytes, const unsigned long long* seg_s1,
                             const unsigned long long* seg_s2, unsigned long long* seg_off, uint8_t* files,
                             unsigned long long* file_bytes) {
    const int f = blockIdx.x, t = threadIdx.x;
    __shared__ unsigned long long s_part[256];
    __shared__ unsigned long long s_carry;
    __shared__ unsigned long long s_adler[2][256];
    if (t == 0) s_carry = 0;
    __syncthreads();
    // exclusive scan of the coded segment sizes, 256 at a time
    for (int base = 0; base < g.nseg; base += 256) {
        const int s = base + t;
        const unsigned long long v = s < g.nseg ? seg_bytes[size_t(f) * g.nseg + s] : 0;
        s_part[t] = v;
        __syncthreads();
        for (int o = 1; o < 256; o <<= 1) {
            const unsigned long long add = t >= o ? s_part[t - o] : 0;
            __syncthreads();
            s_part[t] += add;
            __syncthreads();
        }
        if (s < g.nseg) seg_off[size_t(f) * g.nseg + s] = s_carry + s_part[t] - v;
        __syncthreads();
        if (t == 255) s_carry += s_part[255];
        __syncthreads();
    }
    const unsigned long long D = s_carry;
    // Adler-32 of the zlib input: A = 1 + sum b, B = U + sum_s [s2_s + (U - o_s - l_s) s1_s]
    const unsigned long long M = 65521;
    unsigned long long a = 0, b = 0;
    for (int s = t; s < g.nseg; s += 256) {
        const unsigned long long o = (unsigned long long)s * kSeg;
        const unsigned long long l = std::min<unsigned long long>(kSeg, g.U - o);
        const unsigned long long s1 = seg_s1[size_t(f) * g.nseg + s], s2 = seg_s2[size_t(f) * g.nseg + s];
        a = (a + s1 % M) % M;
        b = (b + s2 % M + ((g.U - o - l) % M) * (s1 % M)) % M;
    }
    s_adler[0][t] = a;
    s_adler[1][t] = b;
    __syncthreads();
    uint8_t* file = files + size_t(f) * g.fstride;
    if (t == 0) {
        unsigned long long A = 1, B = g.U % M;
        for (int i = 0; i < 256; ++i) A = (A + s_adler[0][i]) % M, B = (B + s_adler[1][i]) % M;
        for (int i = 0; i < kPrefix; ++i) file[i] = head.bytes[i];
        put_be32(file + 33, uint32_t(2 + D + 4));   // IDAT data length
        uint8_t* tail = file + kPrefix + D;
        put_be32(tail, uint32_t((B << 16) | A));
        // tail + 4: the IDAT CRC (k_png_crc_final); then IEND
        const uint8_t iend[12] = {0, 0, 0, 0, 'I', 'E', 'N', 'D', 0xAE, 0x42, 0x60, 0x82};
        for (int i = 0; i < 12; ++i) tail[8 + i] = iend[i];
        file_bytes[f] = kPrefix + D + kSuffix;
    }
}

__global__ void k_png_gather(PngGeom g, const uint8_t* __restrict__ slots, const uint32_t* seg_bytes,
                             const unsigned long long* seg_off, uint8_t* __restrict__ files) {
    const int seg = blockIdx.x, f = blockIdx.y;
    const size_t k = size_t(f) * g.nseg + seg;
    const uint8_t* src = slots + k * kSlot;
    uint8_t* dst = files + size_t(f) * g.fstride + kPrefix + seg_off[k];
    const int nb = int(seg_bytes[k]);
    for (int i = threadIdx.x; i < nb; i += blockDim.x) dst[i] = src[i];
}

// Raw (no pre/post inversion) CRC of each 128 KiB block of every file's IDAT type + data,
// the range front-padded with zeros to whole blocks (zeros before any data leave a zero
// register unchanged, so the padding does not alter the result).
__global__ void __launch_bounds__(kCrcThreads) k_png_crc(PngGeom g, CrcTables tb, const uint8_t* __restrict__ files,
                                                         const unsigned long long* file_bytes, uint32_t* blk_crc) {
    __shared__ uint32_t table[256];
    __shared__ uint32_t s_warp[kCrcThreads / 32];
    const int blk = blockIdx.x, f = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const long long L = (long long)file_bytes[f] - kIdatType - 16;   // "IDAT" .. Adler-32
    const long long nblk = (L + kCrcSpan - 1) / kCrcSpan;
    if (blk >= nblk) return;
    if (t < 256) {
        uint32_t c = uint32_t(t);
        for (int k = 0; k < 8; ++k) c = (c >> 1) ^ ((c & 1u) ? kPoly : 0u);
        table[t] = c;
    }
    __syncthreads();
    const long long pad = nblk * kCrcSpan - L;
    const uint8_t* base = files + size_t(f) * g.fstride + kIdatType;
    const long long v0 = (long long)blk * kCrcSpan + (long long)t * kCrcChunk;   // virtual offset
    uint32_t c = 0;
    for (int i = 0; i < kCrcChunk; ++i) {
        const long long v = v0 + i;
        const uint32_t b = v >= pad ? base[v - pad] : 0u;
        c = table[(c ^ b) & 0xFF] ^ (c >> 8);
    }
    // warp tree: a left group followed by a right group of 256 * 2^k bytes each
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const uint32_t other = __shfl_xor_sync(0xffffffffu, c, 1 << k);
        const bool left = !(lane & (1 << k));
        c = left ? (gf_mul(c, tb.lane[k]) ^ other) : (gf_mul(other, tb.lane[k]) ^ c);
    }
    if (lane == 0) s_warp[warp] = c;
    __syncthreads();
    if (t == 0) {
        uint32_t acc = s_warp[0];
        for (int w = 1; w < kCrcThreads / 32; ++w) acc = gf_mul(acc, tb.warp) ^ s_warp[w];
        blk_crc[size_t(f) * g.crc_blocks + blk] = acc;
    }
}

__global__ void k_png_crc_final(PngGeom g, CrcTables tb, const uint32_t* blk_crc,
                                const unsigned long long* file_bytes, uint8_t* files) {
    __shared__ uint32_t s_x[8];
    const int f = blockIdx.x, t = threadIdx.x;
    const long long L = (long long)file_bytes[f] - kIdatType - 16;
    const long long nblk = (L + kCrcSpan - 1) / kCrcSpan;
    uint32_t x = 0;
    for (long long b = t; b < nblk; b += blockDim.x)
        x ^= gf_mul(blk_crc[size_t(f) * g.crc_blocks + b], gf_pow((unsigned long long)(nblk - 1 - b), tb.block_pow));
    for (int o = 16; o > 0; o >>= 1) x ^= __shfl_xor_sync(0xffffffffu, x, o);
    if ((t & 31) == 0) s_x[t >> 5] = x;
    __syncthreads();
    if (t == 0) {
        uint32_t r = 0;
        for (int w = 0; w < int(blockDim.x / 32); ++w) r ^= s_x[w];
        // standard CRC-32: register starts at all ones (advanced over L bytes), result inverted
        const uint32_t crc = r ^ gf_mul(0xFFFFFFFFu, gf_pow((unsigned long long)L, tb.byte_pow)) ^ 0xFFFFFFFFu;
        put_be32(files + size_t(f) * g.fstride + kIdatType + L, crc);
    }
}

// ---- host ------------------------------------------------------------------------------------

uint32_t host_crc32(const uint8_t* p, size_t n) {
    uint32_t c = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; ++i) {
        c ^= p[i];
        for (int k = 0; k < 8; ++k) c = (c >> 1) ^ ((c & 1u) ? kPoly : 0u);
    }
    return c ^ 0xFFFFFFFFu;
}

void put_be32_host(uint8_t* p, uint32_t v) {
    p[0] = uint8_t(v >> 24), p[1] = uint8_t(v >> 16), p[2] = uint8_t(v >> 8), p[3] = uint8_t(v);
}

PngGeom geometry(int n, int h, int w) {
    PngGeom g{};
    g.n = n;
    g.h = h;
    g.w = w;
    g.row = 3LL * w + 1;
    g.U = g.row * h;
    g.ustride = (g.U + 15) / 16 * 16;
    g.nseg = int((g.U + kSeg - 1) / kSeg);
    const long long bound = kPrefix + g.U + 5LL * g.nseg + kSuffix;
    g.fstride = (bound + 15) / 16 * 16;
    const long long L = bound - kIdatType - 16;
    g.crc_blocks = int((L + kCrcSpan - 1) / kCrcSpan);
    return g;
}

CrcTables crc_tables() {
    CrcTables tb{};
    tb.byte_pow[0] = 0x80000000u >> 8;   // x^8
    for (int j = 1; j < 40; ++j) tb.byte_pow[j] = gf_mul(tb.byte_pow[j - 1], tb.byte_pow[j - 1]);
    tb.block_pow[0] = gf_pow((unsigned long long)kCrcSpan, tb.byte_pow);
    for (int j = 1; j < 32; ++j) tb.block_pow[j] = gf_mul(tb.block_pow[j - 1], tb.block_pow[j - 1]);
    for (int k = 0; k < 5; ++k) tb.lane[k] = gf_pow((unsigned long long)kCrcChunk << k, tb.byte_pow);
    tb.warp = gf_pow(32ull * kCrcChunk, tb.byte_pow);
    return tb;
}

PngHead png_head(int h, int w) {
    PngHead hd{};
    const uint8_t sig[8] = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1A, '\n'};
    std::memcpy(hd.bytes, sig, 8);
    uint8_t* ihdr = hd.bytes + 8;
    put_be32_host(ihdr, 13);
    std::memcpy(ihdr + 4, "IHDR", 4);
    put_be32_host(ihdr + 8, uint32_t(w));
    put_be32_host(ihdr + 12, uint32_t(h));
    ihdr[16] = 8;   // bit depth
    ihdr[17] = 2;   // colour type: truecolour (RGB)
    ihdr[18] = ihdr[19] = ihdr[20] = 0;   // deflate, adaptive filtering, no interlace
    put_be32_host(ihdr + 21, host_crc32(ihdr + 4, 17));
    std::memcpy(hd.bytes + 37, "IDAT", 4);
    hd.bytes[41] = 0x78;   // zlib: deflate, 32 KiB window
    hd.bytes[42] = 0x01;   // no dictionary, check bits: (0x78 << 8 | 0x01) % 31 == 0
    return hd;
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

// Per-device scratch, grown on demand and kept; a call holds the device's lock throughout.
struct Scratch {
    std::mutex mu;
    void* p = nullptr;
    size_t bytes = 0;
};
std::mutex g_scratch_mu;
std::map<int, std::unique_ptr<Scratch>> g_scratch;

Scratch& scratch_for(int device) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    auto& s = g_scratch[device];
    if (!s) s = std::make_unique<Scratch>();
    return *s;
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

uint64_t png_bound(int h, int w) {
    require(h >= 1 && w >= 1, "image is empty");
    const PngGeom g = geometry(1, h, w);
    return uint64_t(kPrefix + g.U + 5LL * g.nseg + kSuffix);
}

void png_encode(const void* src, int kind, int n, int h, int w, bool host_io, int device, uint8_t* out,
                uint64_t capacity, uint64_t* sizes, cudaStream_t stream) {
    require(src != nullptr && out != nullptr && sizes != nullptr, "null pointer");
    require(kind == 0 || kind == 1, "unknown frame kind");
    require(n >= 1 && h >= 1 && w >= 1, "image is empty");
    require(w <= kMaxWidth, "PNG encoder: width above 32768");
    const PngGeom g = geometry(n, h, w);
    require(g.U < (1LL << 31) - kSeg, "PNG encoder: frame too large");
    ScopedDevice guard(device);
    Scratch& sc = scratch_for(device);
    std::lock_guard<std::mutex> lk(sc.mu);
    const size_t in_bytes = size_t(n) * h * w * 3 * (kind ? 4 : 1);
    const size_t segs = size_t(n) * g.nseg;
    const size_t b_in = host_io ? align256(in_bytes) : 0, b_filt = align256(size_t(n) * g.ustride),
                 b_slots = align256(segs * kSlot), b_files = align256(size_t(n) * g.fstride),
                 b_tok = align256(segs * size_t(kSeg) * 4), b_seg = align256(segs * 4), b_off = align256(segs * 8), b_s = align256(segs * 8),
                 b_fb = align256(size_t(n) * 8), b_crc = align256(size_t(n) * g.crc_blocks * 4);
    const size_t need = b_in + b_filt + b_slots + b_tok + b_files + b_seg + b_off + 2 * b_s + b_fb + b_crc;
    if (sc.bytes < need) {
        if (sc.p) {
            AEISU_CUDA(cudaStreamSynchronize(stream));
            AEISU_CUDA(cudaFree(sc.p));
            sc.p = nullptr;
            sc.bytes = 0;
        }
        AEISU_CUDA(cudaMalloc(&sc.p, need));
        sc.bytes = need;
    }
    uint8_t* q = static_cast<uint8_t*>(sc.p);
    auto take = [&](size_t b) { uint8_t* r = q; q += b; return r; };
    const void* dsrc = src;
    if (host_io) {
        uint8_t* d = take(b_in);
        AEISU_CUDA(cudaMemcpyAsync(d, src, in_bytes, cudaMemcpyHostToDevice, stream));
        dsrc = d;
    }
    uint8_t* filt = take(b_filt);
    uint8_t* slots = take(b_slots);
    uint32_t* tokens = reinterpret_cast<uint32_t*>(take(b_tok));
    uint8_t* files = take(b_files);
    uint32_t* seg_bytes = reinterpret_cast<uint32_t*>(take(b_seg));
    auto* seg_off = reinterpret_cast<unsigned long long*>(take(b_off));
    auto* seg_s1 = reinterpret_cast<unsigned long long*>(take(b_s));
    auto* seg_s2 = reinterpret_cast<unsigned long long*>(take(b_s));
    auto* file_bytes = reinterpret_cast<unsigned long long*>(take(b_fb));
    uint32_t* blk_crc = reinterpret_cast<uint32_t*>(take(b_crc));

    const int filt_smem = 6 * w;
    if (filt_smem > 48 * 1024)
        AEISU_CUDA(cudaFuncSetAttribute(k_png_filter, cudaFuncAttributeMaxDynamicSharedMemorySize, filt_smem));
    k_png_filter<<<dim3(h, n), kFiltThreads, filt_smem, stream>>>(dsrc, kind, g, filt);
    AEISU_CUDA(cudaGetLastError());
    AEISU_CUDA(cudaFuncSetAttribute(k_png_deflate, cudaFuncAttributeMaxDynamicSharedMemorySize, kDefSmem));
    k_png_deflate<<<dim3(g.nseg, n), kDefThreads, kDefSmem, stream>>>(g, filt, slots, tokens, seg_bytes, seg_s1,
                                                                     seg_s2);
    AEISU_CUDA(cudaGetLastError());
    k_png_layout<<<n, 256, 0, stream>>>(g, png_head(h, w), seg_bytes, seg_s1, seg_s2, seg_off, files, file_bytes);
    AEISU_CUDA(cudaGetLastError());
    k_png_gather<<<dim3(g.nseg, n), 256, 0, stream>>>(g, slots, seg_bytes, seg_off, files);
    AEISU_CUDA(cudaGetLastError());
    static const CrcTables tables = crc_tables();
    k_png_crc<<<dim3(g.crc_blocks, n), kCrcThreads, 0, stream>>>(g, tables, files, file_bytes, blk_crc);
    AEISU_CUDA(cudaGetLastError());
    k_png_crc_final<<<n, 256, 0, stream>>>(g, tables, blk_crc, file_bytes, files);
    AEISU_CUDA(cudaGetLastError());
    std::vector<unsigned long long> fb(n);
    AEISU_CUDA(cudaMemcpyAsync(fb.data(), file_bytes, size_t(n) * 8, cudaMemcpyDeviceToHost, stream));
    AEISU_CUDA(cudaStreamSynchronize(stream));
    uint64_t total = 0;
    for (int f = 0; f < n; ++f) {
        sizes[f] = fb[f];
        total += fb[f];
    }
    if (total > capacity)
        fail(AEISU_ERR_INVALID_ARG, "output buffer too small for the PNG files: need " + std::to_string(total) +
                                        " bytes (sizes[] holds each file's size)");
    uint64_t at = 0;
    for (int f = 0; f < n; ++f) {
        AEISU_CUDA(cudaMemcpyAsync(out + at, files + size_t(f) * g.fstride, fb[f], cudaMemcpyDefault, stream));
        at += fb[f];
    }
    AEISU_CUDA(cudaStreamSynchronize(stream));
}

int png_launches_per_call() { return 6; }

}  // namespace aeisu
