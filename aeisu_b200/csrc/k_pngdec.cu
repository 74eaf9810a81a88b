// PNG ingress on the GPU: the decode half of read_rgb (aeisu/runtime.py:17-20), which opens an
// image file with PIL, converts it to RGB and takes its uint8 HWC pixels.
//
// Host: chunk parsing and checks as PIL makes them (signature, IHDR, PLTE, the CRC-32 of every
// chunk before the image data, the zlib header), IDAT payloads concatenated per file into one
// upload.  GPU: one CTA of two warps per file (k_png_decode):
//   warp 0  decodes the file's deflate stream (RFC 1951: stored, fixed and dynamic Huffman
//           blocks) in lockstep into a 32 KiB shared-memory window, the lanes sharing match
//           copies, stored blocks and table fills, and writes every 8 KiB of output to the
//           scratch buffer, publishing its progress in shared memory; a deflate stream is
//           sequential, so the parallelism is across files.
//   warp 1  follows it: once a group of 32 rows is inflated, their scanline filters (PNG spec
//           section 9: None, Sub, Up, Average, Paeth) are undone one row per lane as a
//           wavefront (each lane one pixel behind the lane above it) over rows staged in shared
//           memory by cp.async, the pixels are converted to RGB (grey replicated, palette looked
//           up, alpha dropped, as PIL's convert("RGB") does) and written as uint8 HWC, and the
//           Adler-32 of the inflated bytes is gathered and checked against the zlib trailer.
// Supported: 8-bit samples, colour types 0, 2, 3, 4 and 6, no interlacing; other files are
// rejected with AEISU_ERR_UNSUPPORTED.  Every read of the compressed stream is bounded by its
// length and every write by the expected image size; a malformed stream sets the file's error
// code and ends its decode, so no loop runs unbounded; warp 1's waits for warp 0 are bounded
// too (polls with a sleep, then an error status instead of a hang).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "kernels.h"
#include "tc.cuh"

namespace aeisu {
namespace {

constexpr int kWin = 32768, kWinMask = kWin - 1;   // deflate window (RFC 1951 2)
constexpr int kFlush = 8192;                       // output bytes written to global per flush
constexpr int kFastBits = 10;                      // Huffman codes up to 10 bits decode by one lookup
constexpr int kMaxLitLen = 288, kMaxDist = 32;

// Per-file status written by the kernels: error code (0 ok), bytes inflated, the zlib trailer's
// Adler-32, the Adler-32 of the inflated bytes.
enum DecErr : int {
    kDecOk = 0, kDecBadBlock = 1, kDecBadCode = 2, kDecBadDistance = 3, kDecOverflow = 4, kDecTruncated = 5,
    kDecShort = 6, kDecAdler = 7, kDecBadFilter = 8, kDecBadPalette = 9, kDecWaitLimit = 10
};
struct DecStatus {
    int error;
    unsigned int adler_stored, adler_computed;
    int check_adler;                     // 0: the stream held more than the image, or no trailer
    unsigned long long produced;
    unsigned long long sum, weighted;    // sum of the inflated bytes x_i, and of (i mod 65521) x_i
};

struct DecFile {
    unsigned long long in_off, in_len;   // deflate stream + 4-byte Adler trailer in the input buffer
    unsigned long long out_off;          // inflated (filtered) scanlines in the scratch buffer
    int color, bpp, npal;                // PNG colour type, bytes per pixel, palette entries
    int pal_off;                         // offset of the palette (3 bytes per entry) in the palette buffer
};

// What a file's inflating warp tells its unfiltering warp, in shared memory: how many inflated
// bytes are in the scratch buffer, and, once it is done, its result.
struct Handoff {
    unsigned flushed;
    int done, err, check;
    unsigned stored, produced;
};

struct DecGeom {
    int n, h, w;
    unsigned long long out_stride;       // bytes of one output frame (h * w * 3)
};

// RFC 1951 3.2.5: base values and extra bits of the length symbols 257..285 and of the distance
// symbols 0..29.
__constant__ uint16_t c_len_base[29] = {3, 4, 5, 6, 7, 8, 9, 10, 11, 13, 15, 17, 19, 23, 27, 31,
                                        35, 43, 51, 59, 67, 83, 99, 115, 131, 163, 195, 227, 258};
__constant__ uint8_t c_len_extra[29] = {0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 2,
                                        3, 3, 3, 3, 4, 4, 4, 4, 5, 5, 5, 5, 0};
__constant__ uint16_t c_dist_base[30] = {1, 2, 3, 4, 5, 7, 9, 13, 17, 25, 33, 49, 65, 97, 129, 193,
                                         257, 385, 513, 769, 1025, 1537, 2049, 3073, 4097, 6145,
                                         8193, 12289, 16385, 24577};
__constant__ uint8_t c_dist_extra[30] = {0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6, 6,
                                         7, 7, 8, 8, 9, 9, 10, 10, 11, 11, 12, 12, 13, 13};
// order of the code-length code lengths in a dynamic block header (RFC 1951 3.2.7)
__constant__ uint8_t c_cl_order[19] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};

// LSB-first bit reader over one file's stream, 32 bits per load (the stream starts 16-byte
// aligned and is followed by zero padding to the next 16 bytes).  Words past the end read as
// zero and are counted, so that a stream that runs out is detected after the fact
// (consumed() > length).  Every lane of the warp holds the same reader state.
struct BitReader {
    const uint32_t* base;
    const uint32_t* wp;
    const uint32_t* wend;
    uint64_t buf;
    int cnt;
    __device__ __forceinline__ void refill() {   // leaves at least 32 bits
        if (cnt <= 32) {
            const uint32_t v = wp < wend ? __ldg(wp) : 0u;
            ++wp;
            buf |= uint64_t(v) << cnt;
            cnt += 32;
        }
    }
    __device__ __forceinline__ uint32_t peek() const { return uint32_t(buf); }
    __device__ __forceinline__ void skip(int n) {
        buf >>= n;
        cnt -= n;
    }
    __device__ __forceinline__ uint32_t bits(int n) {   // n <= 32
        if (cnt < n) refill();
        const uint32_t v = uint32_t(buf & ((1ull << n) - 1));
        skip(n);
        return v;
    }
    __device__ long long consumed() const { return (long long)(wp - base) * 32 - cnt; }
    __device__ void seek_byte(unsigned long long off) {   // continue at byte `off` of the stream
        wp = base + off / 4;
        const uint32_t v = wp < wend ? __ldg(wp) : 0u;
        ++wp;
        const int sh = int(off % 4) * 8;
        buf = uint64_t(v >> sh);
        cnt = 32 - sh;
    }
};

// Decoded-symbol entries (32 bits): code length in bits 0-4 (lookup-table entries only), extra
// bits in 5-8, kind in 9-10, value in 16-31.  Kinds: 0 not a valid symbol (or, in the lookup
// table, a code longer than kFastBits), 1 literal byte / code-length symbol, 2 length or
// distance (value = base, RFC 1951 3.2.5), 3 end of block.
enum : uint32_t { kKindMask = 3u << 9, kLiteral = 1u << 9, kCopy = 2u << 9, kEnd = 3u << 9 };
enum HuffMode { kCodeLengths, kLitLen, kDistance };

__device__ __forceinline__ uint32_t symbol_entry(int s, HuffMode mode) {
    if (mode == kCodeLengths) return kLiteral | (uint32_t(s) << 16);
    if (mode == kDistance)
        return s < 30 ? kCopy | (uint32_t(c_dist_extra[s]) << 5) | (uint32_t(c_dist_base[s]) << 16) : 0u;
    if (s < 256) return kLiteral | (uint32_t(s) << 16);
    if (s == 256) return kEnd;
    if (s <= 285) return kCopy | (uint32_t(c_len_extra[s - 257]) << 5) | (uint32_t(c_len_base[s - 257]) << 16);
    return 0u;
}

// A canonical Huffman code: codes up to kFastBits decode with one lookup, longer ones by walking
// the lengths (count per length, symbols in code order).
struct Huff {
    uint32_t fast[1 << kFastBits];
    uint16_t count[16];
    uint16_t sym[kMaxLitLen];
};

// Builds the code of lengths[0..n) with the whole warp; false (on every lane) for an
// over-subscribed set, or an incomplete one unless `lone` and it is a single one-bit code (zlib's
// inflate allows that for literal/length and distance codes, not for the code-length code).  An
// all-zero set gives a code that decodes nothing (a block without matches needs no distances).
// Lane 0 counts the lengths and assigns the codes (bit-reversed into `rev`); all lanes fill the
// lookup table, one symbol per lane.
__device__ bool huff_build(Huff& hf, uint16_t* rev, const uint8_t* len, int n, bool lone, HuffMode mode, int lane) {
    __syncwarp();   // len[] was written by lane 0
    int ok = 1;
    if (lane == 0) {
        for (int l = 0; l < 16; ++l) hf.count[l] = 0;
        int maxlen = 0;
        for (int s = 0; s < n; ++s) {
            hf.count[len[s]]++;
            maxlen = max(maxlen, int(len[s]));
        }
        hf.count[0] = 0;
        int left = 1;
        for (int l = 1; l < 16; ++l) {
            left = (left << 1) - hf.count[l];
            if (left < 0) ok = 0;
        }
        if (maxlen > 0 && left > 0 && (!lone || maxlen != 1)) ok = 0;
        if (ok && maxlen > 0) {
            uint16_t offs[16], next[16];
            offs[1] = 0;
            for (int l = 1; l < 15; ++l) offs[l + 1] = uint16_t(offs[l] + hf.count[l]);
            int code = 0;
            for (int l = 1; l < 16; ++l) {
                code = (code + hf.count[l - 1]) << 1;
                next[l] = uint16_t(code);
            }
            for (int s = 0; s < n; ++s) {
                const int l = len[s];
                if (!l) continue;
                hf.sym[offs[l]++] = uint16_t(s);
                rev[s] = uint16_t(__brev(unsigned(next[l]++)) >> (32 - l));
            }
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    for (int i = lane; i < (1 << kFastBits); i += 32) hf.fast[i] = 0;
    __syncwarp();
    if (ok)
        for (int s = lane; s < n; s += 32) {
            const int l = len[s];
            if (l && l <= kFastBits) {
                const uint32_t e = uint32_t(l) | symbol_entry(s, mode);
                for (int i = rev[s]; i < (1 << kFastBits); i += 1 << l) hf.fast[i] = e;
            }
        }
    __syncwarp();
    return ok != 0;
}

// Codes longer than kFastBits (and bit patterns the code does not contain): canonical decode,
// one bit at a time (the codes of length l are first .. first + count - 1).  Returns the
// symbol's entry with code length 0 (its bits are consumed), or 0 for no symbol.
__device__ __forceinline__ uint32_t huff_slow(BitReader& br, const Huff& hf, HuffMode mode) {
    int code = 0, first = 0, index = 0;
    for (int l = 1; l < 16; ++l) {
        code |= int(br.bits(1));
        const int c = hf.count[l];
        if (unsigned(code - first) < unsigned(c)) return symbol_entry(hf.sym[index + code - first], mode);
        index += c;
        first = (first + c) << 1;
        code <<= 1;
    }
    return 0u;
}

// Next symbol's entry (kind 0: invalid); the reader must hold at least 15 bits.
__device__ __forceinline__ uint32_t huff_decode(BitReader& br, const Huff& hf, HuffMode mode) {
    const uint32_t e = hf.fast[br.peek() & ((1u << kFastBits) - 1)];
    if (e & kKindMask) {
        br.skip(int(e & 31));
        return e;
    }
    return huff_slow(br, hf, mode);
}

// Output side of the inflater: a 32 KiB window in shared memory, written through to global
// memory by the whole warp every kFlush bytes (the window always holds the last 32 KiB, and at
// most kFlush + 258 bytes are not yet written out).  produced and flushed are the same on
// every lane; flushed is a multiple of 16 until the final flush.
struct Window {
    uint8_t* win;
    uint8_t* out;
    const uint8_t* mod;   // mod[32 * d + lane] = lane % d for 1 <= d < 32
    Handoff* ho;          // progress, published after every flush
    unsigned produced, flushed, limit;
    unsigned next;        // the next event: min(flushed + kFlush, limit)
    __device__ void flush(unsigned upto, int lane) {
        __syncwarp();
        // loops with the same trip count on every lane (the body predicated), so the warp
        // never splits
        const unsigned a = flushed, body = a + ((upto - a) & ~15u);
        for (unsigned i0 = a; i0 < body; i0 += 512) {
            const unsigned i = i0 + 16u * lane;
            if (i < body) *reinterpret_cast<uint4*>(out + i) = *reinterpret_cast<const uint4*>(win + (i & kWinMask));
        }
        for (unsigned i0 = body; i0 < upto; i0 += 32) {
            const unsigned i = i0 + lane;
            if (i < upto) out[i] = win[i & kWinMask];
        }
        flushed = upto;
        next = min(flushed + unsigned(kFlush), limit);
        __threadfence_block();   // this lane's stores, before the progress the other warp reads
        __syncwarp();
        if (lane == 0) *reinterpret_cast<volatile unsigned*>(&ho->flushed) = upto;
    }
    // Adds n bytes; true when the image is complete (produced == limit).  One compare against
    // `next` in the common case.
    __device__ __forceinline__ bool advance(unsigned n, int lane) {
        produced += n;
        if (produced < next) return false;
        if (produced - flushed >= unsigned(kFlush)) flush(produced & ~unsigned(kFlush - 1), lane);
        return produced == limit;
    }
    __device__ __forceinline__ bool literal(uint32_t v, int lane) {   // the caller keeps produced < limit
        if (lane == 0) win[produced & kWinMask] = uint8_t(v);
        return advance(1, lane);
    }
    // n bytes from d back (1 <= d <= produced, d <= 32 KiB); the caller keeps produced + n <= limit.
    // Byte k of the copy equals byte k % d of the source.  d >= n: every source byte exists
    // before the copy (one pass).  32 <= d < n: rounds of 32 bytes, each reading only bytes
    // written before the round.  d < 32: each lane reads the source pattern.
    __device__ __forceinline__ void match(int n, int d, int lane) {
        __syncwarp();   // literals written by lane 0
        const unsigned src = produced - unsigned(d);
        if (d >= n) {
            for (int k0 = 0; k0 < n; k0 += 32) {
                const int k = k0 + lane;
                if (k < n) win[(produced + k) & kWinMask] = win[(src + k) & kWinMask];
            }
        } else if (d >= 32) {
            for (int k0 = 0; k0 < n; k0 += 32) {
                const int k = k0 + lane;
                const uint8_t v = k < n ? win[(src + k) & kWinMask] : 0;
                __syncwarp();
                if (k < n) win[(produced + k) & kWinMask] = v;
                __syncwarp();
            }
        } else {
            int m = mod[32 * d + lane];
            const int step = mod[32 * d + 31] + 1 == d ? 0 : mod[32 * d + 31] + 1;   // 32 % d
            for (int k0 = 0; k0 < n; k0 += 32) {
                const int k = k0 + lane;
                if (k < n) win[(produced + k) & kWinMask] = win[(src + m) & kWinMask];
                m += step;
                if (m >= d) m -= d;
            }
        }
        __syncwarp();
    }
};

constexpr int kInflateSmem = kWin + 2 * int(sizeof(Huff)) + 320 + 2 * kMaxLitLen + 32 * 32 + 64;

// End of the stream, as PIL (through zlib) reads it: the image is complete once h scanlines are
// inflated; a stream that would inflate more stops there (the rest is not read, its Adler-32 not
// checked); a stream whose last block ends exactly at the image is checked against its Adler-32
// trailer when the trailer is present, and taken without a check when the stream ends before it
// (or before its last block, or inside a block header, once the image is complete).
// The whole warp runs one file's decode in lockstep: every lane decodes the same symbols (the
// table lookups broadcast), and the lanes share the byte work (match copies, stored blocks,
// flushes, table fills).
__device__ void inflate_file(const uint8_t* __restrict__ in, const DecFile& fd, uint8_t* __restrict__ scratch,
                             const DecGeom& g, uint8_t* smem, Handoff* ho, int lane) {
    uint8_t* win = smem;
    Huff& lit = *reinterpret_cast<Huff*>(smem + kWin);
    Huff& dist = *reinterpret_cast<Huff*>(smem + kWin + sizeof(Huff));
    uint8_t* lens = smem + kWin + 2 * sizeof(Huff);   // code lengths of one block header (<= 320)
    uint16_t* rev = reinterpret_cast<uint16_t*>(lens + 320);   // bit-reversed codes while building
    uint8_t* mod = lens + 320 + 2 * kMaxLitLen;                // mod[32 * d + lane] = lane % d
    for (int d = 1; d < 32; ++d) mod[32 * d + lane] = uint8_t(lane % d);
    const unsigned expect = unsigned(g.h) * (1u + unsigned(g.w) * unsigned(fd.bpp));
    const long long avail = (long long)fd.in_len * 8;   // bits of the stream, trailer included
    const uint8_t* src = in + fd.in_off;
    const uint32_t* words = reinterpret_cast<const uint32_t*>(src);
    BitReader br{words, words, words + (fd.in_len + 3) / 4, 0ull, 0};
    Window wo{win, scratch + fd.out_off, mod, ho, 0u, 0u, expect, min(unsigned(kFlush), expect)};
    int err = kDecOk;
    bool last = false, more = false;   // more: the stream holds data past the image
    long long full_bits = -1;          // bits consumed when the image became complete
    __syncwarp();
    while (!last && !more && err == kDecOk) {
        if (wo.produced == wo.limit && br.consumed() >= avail) break;   // complete, stream ends early
        last = br.bits(1) != 0;
        const int type = int(br.bits(2));
        if (type == 0) {   // stored: byte-aligned LEN, NLEN, LEN raw bytes
            br.bits(br.cnt & 7);
            const uint32_t len = br.bits(16), nlen = br.bits(16);
            if ((len ^ 0xFFFFu) != nlen) { err = kDecBadBlock; break; }
            const unsigned long long pos = (unsigned long long)br.consumed() / 8;
            const unsigned room = wo.limit - wo.produced;
            const unsigned copy = room < len ? room : len;
            for (unsigned done = 0; done < copy;) {   // pieces of at most kFlush bytes
                const unsigned piece = min(copy - done, unsigned(kFlush));
                for (unsigned k0 = 0; k0 < piece; k0 += 32) {
                    const unsigned k = k0 + lane;
                    const unsigned long long at = pos + done + k;
                    if (k < piece) win[(wo.produced + k) & kWinMask] = at < fd.in_len ? src[at] : 0;
                }
                wo.advance(piece, lane);
                done += piece;
            }
            if (copy < len) { more = true; break; }
            br.seek_byte(pos + len);
            if (wo.produced == wo.limit && full_bits < 0) full_bits = (long long)(pos + len) * 8;
            if (wo.produced < wo.limit && br.consumed() > avail) err = kDecTruncated;
            continue;
        }
        if (type == 3) { err = kDecBadBlock; break; }
        if (type == 1) {   // fixed codes (RFC 1951 3.2.6)
            for (int s = lane; s < kMaxLitLen; s += 32) lens[s] = s < 144 ? 8 : s < 256 ? 9 : s < 280 ? 7 : 8;
            huff_build(lit, rev, lens, kMaxLitLen, true, kLitLen, lane);
            for (int s = lane; s < 32; s += 32) lens[s] = 5;   // 32 codes, of which 30 and 31 never occur
            huff_build(dist, rev, lens, 32, true, kDistance, lane);
        } else {           // dynamic codes (RFC 1951 3.2.7)
            const int hlit = int(br.bits(5)) + 257, hdist = int(br.bits(5)) + 1, hclen = int(br.bits(4)) + 4;
            if (hlit > 286 || hdist > 30) { err = kDecBadBlock; break; }
            uint8_t cl[19];
            for (int i = 0; i < 19; ++i) cl[i] = 0;
            for (int i = 0; i < hclen; ++i) cl[c_cl_order[i]] = uint8_t(br.bits(3));
            if (lane == 0)
                for (int i = 0; i < 19; ++i) lens[i] = cl[i];
            if (!huff_build(lit, rev, lens, 19, false, kCodeLengths, lane)) { err = kDecBadCode; break; }
            int i = 0, prev = 0;
            while (i < hlit + hdist) {
                if (br.cnt < 32) br.refill();
                const uint32_t e = huff_decode(br, lit, kCodeLengths);
                if (!(e & kKindMask)) { err = kDecBadCode; break; }
                const int sym = int(e >> 16);
                if (sym < 16) {
                    if (lane == 0) lens[i] = uint8_t(sym);
                    prev = sym;
                    ++i;
                    continue;
                }
                int rep = 0, val = 0;
                if (sym == 16) {
                    if (i == 0) { err = kDecBadCode; break; }
                    val = prev;
                    rep = 3 + int(br.bits(2));
                } else if (sym == 17) {
                    rep = 3 + int(br.bits(3));
                } else {
                    rep = 11 + int(br.bits(7));
                }
                if (i + rep > hlit + hdist) { err = kDecBadCode; break; }
                for (int k = lane; k < rep; k += 32) lens[i + k] = uint8_t(val);   // rep <= 138
                prev = val;
                i += rep;
            }
            if (err != kDecOk) break;
            __syncwarp();
            if (lens[256] == 0) { err = kDecBadCode; break; }   // the block could never end
            if (!huff_build(lit, rev, lens, hlit, true, kLitLen, lane) ||
                !huff_build(dist, rev, lens + hlit, hdist, true, kDistance, lane)) {
                err = kDecBadCode;
                break;
            }
        }
        bool complete = wo.produced == wo.limit, ended = false;
        while (!complete) {   // the block's symbols, until its end or the image's
            if (br.cnt < 32) br.refill();   // a literal/length code and its extra bits: <= 20 bits
            const uint32_t e = huff_decode(br, lit, kLitLen);
            const uint32_t kind = e & kKindMask;
            if (kind == kLiteral) {
                complete = wo.literal(e >> 16, lane);
                continue;
            }
            if (kind == kEnd) { ended = true; break; }
            if (kind == 0) { err = kDecBadCode; break; }
            const int lx = int((e >> 5) & 15);
            const int len = int(e >> 16) + int(br.peek() & ((1u << lx) - 1));
            br.skip(lx);
            if (br.cnt < 28) br.refill();   // a distance code and its extra bits: <= 28 bits
            const uint32_t de = huff_decode(br, dist, kDistance);
            if (!(de & kKindMask)) { err = kDecBadCode; break; }
            const int dx = int((de >> 5) & 15);
            const int d = int(de >> 16) + int(br.peek() & ((1u << dx) - 1));
            br.skip(dx);
            if (unsigned(d) > wo.produced) { err = kDecBadDistance; break; }   // d <= 32768 always
            const unsigned room = wo.limit - wo.produced;
            const int copy = room < unsigned(len) ? int(room) : len;
            wo.match(copy, d, lane);
            complete = wo.advance(unsigned(copy), lane);
            if (copy < len) more = true;
        }
        if (complete && err == kDecOk) {
            if (full_bits < 0) full_bits = br.consumed();   // the bits that completed the image
            // past the image, as zlib reads on: the block's end, or data the image has no room for
            while (!ended && !more) {
                if (br.cnt < 32) br.refill();
                const uint32_t e = huff_decode(br, lit, kLitLen);
                const uint32_t kind = e & kKindMask;
                if (kind == kEnd) ended = true;
                else if (kind == kLiteral) more = true;
                else if (kind == 0) { err = kDecBadCode; break; }
                else {   // a match: zlib decodes its distance code, then stops for want of room
                    br.skip(int((e >> 5) & 15));   // (before its distance-too-far check)
                    if (br.cnt < 28) br.refill();
                    if (!(huff_decode(br, dist, kDistance) & kKindMask)) { err = kDecBadCode; break; }
                    more = true;
                }
            }
        }
        if (!more && err == kDecOk && wo.produced < wo.limit && br.consumed() > avail) err = kDecTruncated;
    }
    wo.flush(wo.produced, lane);
    // zlib waits for more input where a field runs past the stream's end: once the image is
    // complete, an error found only in the zero bits past the end is no error
    if (err != kDecOk && wo.produced == expect && full_bits >= 0 && full_bits <= avail && br.consumed() > avail)
        err = kDecOk;
    unsigned int stored = 0;
    int check = 0;
    if (err == kDecOk) {
        if (wo.produced != expect) err = br.consumed() > avail ? kDecTruncated : kDecShort;
        else if (full_bits > avail) err = kDecTruncated;
        else if (!more && br.consumed() <= avail) {
            // the zlib trailer: Adler-32, big-endian, at the next byte boundary, if present
            br.bits(br.cnt & 7);
            if (br.consumed() + 32 <= avail) {
                for (int k = 0; k < 4; ++k) stored = (stored << 8) | br.bits(8);
                check = 1;
            }
        }
    }
    if (lane == 0) {
        volatile Handoff* v = ho;
        v->err = err;
        v->check = check;
        v->stored = stored;
        v->produced = wo.produced;
        __threadfence_block();
        v->done = 1;
    }
}

__device__ __forceinline__ int paeth(int a, int b, int c) {
    const int p = a + b - c, pa = abs(p - a), pb = abs(p - b), pc = abs(p - c);
    return (pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c);
}

using tc::cp_async_commit;
using tc::cp_async_wait_group;
using tc::smem_addr;

// 4-byte global -> shared asynchronous copy (both addresses 4-byte aligned).
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(smem_addr(smem)), "l"(gmem) : "memory");
}

// Shared-memory staging of the unfilter: the filtered bytes of a group's 32 rows and of the row
// above it, in chunks of 32 pixels (kUnfBufs chunks in flight: two being read, two loading),
// each row's chunk as the aligned words that cover it (8 * BPP + 1 words: an odd word stride,
// so the 32 lanes' rows fall in different banks); and the RGB output of two chunks.
constexpr int kUnfBufs = 4;
constexpr int kUnfRowWords = 8 * 4 + 1;                    // BPP = 4, the largest
constexpr int kUnfInBytes = kUnfBufs * 33 * 4 * kUnfRowWords;
constexpr int kUnfOutRow = 100;                            // 32 pixels x 3 bytes, odd word stride
constexpr int kUnfOutBytes = 2 * 32 * kUnfOutRow;

// Waits (lane 0 polling, bounded) until the inflating warp has flushed `need` bytes of the
// file: 1 when they are there, 0 when the inflate ended before them (its result decides),
// -1 when the wait gave up.
constexpr unsigned kWaitSpins = 1u << 25;

__device__ int wait_inflated(const Handoff* ho, unsigned long long need, int lane) {
    int r = -1;
    if (lane == 0) {
        const volatile Handoff* v = ho;
        for (unsigned it = 0; it < kWaitSpins; ++it) {
            if (v->flushed >= need) { r = 1; break; }
            if (v->done) { r = v->flushed >= need ? 1 : 0; break; }
            __nanosleep(256);
        }
    }
    r = __shfl_sync(0xffffffffu, r, 0);
    __threadfence_block();   // the inflated bytes, after the progress that announced them
    return r;
}

// One file, BPP bytes per pixel, behind the inflating warp: each group of rows starts once the
// inflate has written all of it.  Rows go in groups of 32, one row per lane, as a wavefront:
// at step t lane r undoes pixel x = t - r of row y0 + r, so the row above's pixels x and x - 1
// are the ones lane r - 1 finished at steps t - 1 and t - 2 (passed by a warp shuffle); lane 0
// reads the row above the group (unfiltered by lane 31 of the previous group and written back
// to the scratch buffer) from the staged chunks.  Steps go in phases of 32: in phase p the
// lanes read chunks p - 1 and p, chunk p + 2 is loading, and chunk p - 1's output is complete
// at the phase's end and written out, one row at a time by the whole warp.  The filter type (a
// lane's own row's) picks the predictor by selects, so the lanes do not diverge.
// On the way, each lane adds up its rows' filtered bytes for the Adler-32 of the stream (RFC
// 1950 8.2) in a form that does not depend on the order: sum x_i and sum (i mod 65521) x_i over
// byte positions i; the warp's totals are returned in sum and weighted (lane 0).
template <int BPP>
__device__ int unfilter_file(const DecFile& fd, uint8_t* rows, const uint8_t* s_pal, const DecGeom& g, uint8_t* dst,
                             uint8_t* s_in, uint8_t* s_out, const Handoff* ho, unsigned long long& sum,
                             unsigned long long& weighted, int lane) {
    constexpr int CB = 32 * BPP, RW = 8 * BPP + 1, RS = 4 * RW;
    const unsigned long long stride = 1ull + (unsigned long long)g.w * BPP;
    const int nchunks = (g.w + 31) / 32, last_phase = (g.w + 30) / 32;
    constexpr unsigned kMod = 65521;
    sum = weighted = 0;
    int result = kDecOk;
    for (int y0 = 0; y0 < g.h; y0 += 32) {
        const int y = y0 + lane;
        const bool active = y < g.h;
        const int rows_here = min(32, g.h - y0);
        const int ready = wait_inflated(ho, (unsigned long long)(y0 + rows_here) * stride, lane);
        if (ready <= 0) {
            result = ready == 0 ? kDecOk : kDecWaitLimit;   // an ended inflate reports its own error
            break;
        }
        const int type = active ? rows[(unsigned long long)y * stride] : 0;
        if (__any_sync(0xffffffffu, type > 4)) {
            result = kDecBadFilter;
            break;
        }
        if (active) {
            sum += unsigned(type);
            weighted += ((unsigned long long)y * stride % kMod) * unsigned(type);
        }
        unsigned pos = unsigned(((unsigned long long)y * stride + 1) % kMod);   // byte position of pixel x, mod 65521
        // byte offset of a row's first data byte inside its staged words
        const int mis = active ? int((unsigned long long)y * stride + 1) & 3 : 0;
        const int mis_above = y0 > 0 ? int((unsigned long long)(y0 - 1) * stride + 1) & 3 : 0;
        auto load = [&](int c) {   // chunk c of rows y0 - 1 .. y0 + rows_here - 1, one commit group
            if (c < nchunks) {
                uint8_t* buf = s_in + (c % kUnfBufs) * 33 * RS;
                for (int slot = y0 > 0 ? -1 : 0; slot < rows_here; ++slot) {
                    const uintptr_t first =
                        uintptr_t(rows + (unsigned long long)(y0 + slot) * stride + 1 + (unsigned long long)c * CB);
                    const uint8_t* al = reinterpret_cast<const uint8_t*>(first & ~uintptr_t(3));
                    uint8_t* srow = buf + (slot < 0 ? 32 : slot) * RS;
                    for (int k0 = 0; k0 < RW; k0 += 32)
                        if (k0 + lane < RW) cp_async4(srow + 4 * (k0 + lane), al + 4 * (k0 + lane));
                }
            }
            cp_async_commit();
        };
        __syncwarp();
        load(0);
        load(1);
        uint32_t cur = 0, left = 0, ul = 0;   // packed pixels: this row's last, its left, above-left
        for (int p = 0; p <= last_phase; ++p) {
            __syncwarp();   // every lane is done with chunk p - 2's buffer
            load(p + 2);
            cp_async_wait_group<2>();
            __syncwarp();   // chunk p (every lane's copies) is in shared memory
            for (int s = 0; s < 32; ++s) {
                // branch-free step: every lane reads (from clamped positions) and computes; only
                // the stores are predicated, so the warp never splits
                const int t = 32 * p + s, x = t - lane;
                const bool valid = active && x >= 0 && x < g.w;
                const int xc = min(max(x, 0), g.w - 1);
                const int c = xc >> 5;
                const uint8_t* buf = s_in + (c % kUnfBufs) * 33 * RS;
                const int o = (xc - 32 * c) * BPP;
                const uint32_t shuffled = __shfl_up_sync(0xffffffffu, cur, 1);
                uint32_t above = 0, res = 0, bsum = 0, jsum = 0;
                const uint8_t* fb = buf + lane * RS + mis + o;
                const uint8_t* ab = buf + 32 * RS + mis_above + o;
#pragma unroll
                for (int j = 0; j < BPP; ++j) above |= uint32_t(ab[j]) << (8 * j);
                const uint32_t up = lane > 0 ? shuffled : (y0 > 0 ? above : 0u);
#pragma unroll
                for (int j = 0; j < BPP; ++j) {
                    const int v = fb[j];
                    bsum += unsigned(v);
                    jsum += unsigned(j * v);
                    const int la = (left >> (8 * j)) & 255, ub = (up >> (8 * j)) & 255, uc = (ul >> (8 * j)) & 255;
                    const int pred = type == 0 ? 0 : type == 1 ? la : type == 2 ? ub : type == 3 ? ((la + ub) >> 1)
                                                                                                : paeth(la, ub, uc);
                    res |= uint32_t((v + pred) & 255) << (8 * j);
                }
                cur = valid ? res : cur;
                left = cur;
                if (valid) {
                    sum += bsum;
                    weighted += (unsigned long long)pos * bsum + jsum;
                    pos += BPP;
                    if (pos >= kMod) pos -= kMod;
                }
                if (valid && lane == 31)   // the next group's row above
#pragma unroll
                    for (int j = 0; j < BPP; ++j)
                        rows[(unsigned long long)y * stride + 1 + (unsigned long long)x * BPP + j] = uint8_t(res >> (8 * j));
                uint32_t rgb;
                if (BPP >= 3) {
                    rgb = res;
                } else if (fd.color == 3) {
                    const int k = res & 255;   // PIL: entries beyond the palette read as black
                    rgb = k < fd.npal ? uint32_t(s_pal[3 * k]) | uint32_t(s_pal[3 * k + 1]) << 8 |
                                            uint32_t(s_pal[3 * k + 2]) << 16
                                      : 0u;
                } else {   // grey, grey + alpha
                    rgb = (res & 255u) * 0x010101u;
                }
                uint8_t* ob = s_out + (c & 1) * 32 * kUnfOutRow + lane * kUnfOutRow + (xc - 32 * c) * 3;
                if (valid) {
                    ob[0] = uint8_t(rgb);
                    ob[1] = uint8_t(rgb >> 8);
                    ob[2] = uint8_t(rgb >> 16);
                }
                ul = up;
            }
            // chunk p - 1 is complete on every row (and, after the last phase, chunk last_phase)
            for (int c = p - 1; c <= (p == last_phase ? min(p, nchunks - 1) : p - 1); ++c) {
                if (c < 0) continue;
                __syncwarp();
                const int n = 3 * min(32, g.w - 32 * c);
                for (int r = 0; r < rows_here; ++r) {
                    uint8_t* orow = dst + ((unsigned long long)(y0 + r) * g.w + 32ull * c) * 3;
                    const uint8_t* ob = s_out + (c & 1) * 32 * kUnfOutRow + r * kUnfOutRow;
                    for (int k0 = 0; k0 < n; k0 += 32)
                        if (k0 + lane < n) orow[k0 + lane] = ob[k0 + lane];
                }
            }
        }
        cp_async_wait_group<0>();
        __syncwarp();   // lane 31's row is read back by the next group
    }
    for (int o = 16; o > 0; o >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        weighted += __shfl_xor_sync(0xffffffffu, weighted, o);
    }
    return result;
}

constexpr int kDecodeSmem = kInflateSmem + kUnfInBytes + kUnfOutBytes + 768 + 64;

// One CTA per file, two warps: warp 0 inflates the file's stream into the scratch buffer; warp
// 1 undoes the scanline filters of each group of 32 rows once warp 0 has written it, converts
// to RGB and checks the Adler-32, so the unfilter runs under the inflate.  Warp 1 writes the
// file's status.
__global__ void __launch_bounds__(64) k_png_decode(const uint8_t* __restrict__ in, const DecFile* __restrict__ files,
                                                   uint8_t* __restrict__ scratch, const uint8_t* __restrict__ palettes,
                                                   DecGeom g, uint8_t* __restrict__ out, DecStatus* status) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* s_in = smem + kInflateSmem;
    uint8_t* s_out = s_in + kUnfInBytes;
    uint8_t* s_pal = s_out + kUnfOutBytes;
    Handoff* ho = reinterpret_cast<Handoff*>(s_pal + 768);
    const int f = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (f >= g.n) return;
    if (threadIdx.x == 0) *ho = Handoff{0u, 0, 0, 0, 0u, 0u};
    __syncthreads();
    const DecFile fd = files[f];
    if (warp == 0) {
        inflate_file(in, fd, scratch, g, smem, ho, lane);
        return;
    }
    for (int i = lane; i < 3 * fd.npal; i += 32) s_pal[i] = palettes[fd.pal_off + i];
    __syncwarp();
    uint8_t* rows = scratch + fd.out_off;
    uint8_t* dst = out + (unsigned long long)f * g.out_stride;
    unsigned long long sum = 0, weighted = 0;
    int err;
    switch (fd.bpp) {
        case 1: err = unfilter_file<1>(fd, rows, s_pal, g, dst, s_in, s_out, ho, sum, weighted, lane); break;
        case 2: err = unfilter_file<2>(fd, rows, s_pal, g, dst, s_in, s_out, ho, sum, weighted, lane); break;
        case 3: err = unfilter_file<3>(fd, rows, s_pal, g, dst, s_in, s_out, ho, sum, weighted, lane); break;
        default: err = unfilter_file<4>(fd, rows, s_pal, g, dst, s_in, s_out, ho, sum, weighted, lane); break;
    }
    // the inflate's result (after the unfilter stopped, or timed out waiting for it)
    if (wait_inflated(ho, ~0ull, lane) < 0 && err == kDecOk) err = kDecWaitLimit;
    if (lane == 0) {
        const volatile Handoff* v = ho;
        DecStatus st{};
        st.error = v->done ? v->err : kDecWaitLimit;
        st.adler_stored = v->stored;
        st.check_adler = v->check;
        st.produced = v->produced;
        st.sum = sum;
        st.weighted = weighted;
        // Adler-32 (RFC 1950 8.2) of the n inflated bytes: a = 1 + sum x_i, b = sum over k of the
        // a after k bytes = n + sum (n - i) x_i = n + n sum x_i - sum i x_i, all mod 65521
        const unsigned long long m = 65521, n = st.produced % m;
        const unsigned long long a = (1 + sum) % m;
        const unsigned long long b = (n + n * (sum % m) + m - weighted % m) % m;
        st.adler_computed = (unsigned int)((b << 16) | a);
        if (st.error == kDecOk) {
            if (err != kDecOk) st.error = err;
            else if (st.check_adler && st.adler_computed != st.adler_stored) st.error = kDecAdler;
        }
        status[f] = st;
    }
}

// ---- host ------------------------------------------------------------------------------------

// CRC-32 (ISO-HDLC, the PNG chunk CRC), eight bytes per step with eight 256-entry tables.
struct Crc8 {
    uint32_t t[8][256];
    Crc8() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c >> 1) ^ ((c & 1u) ? 0xEDB88320u : 0u);
            t[0][i] = c;
        }
        for (int j = 1; j < 8; ++j)
            for (int i = 0; i < 256; ++i) t[j][i] = (t[j - 1][i] >> 8) ^ t[0][t[j - 1][i] & 0xFF];
    }
    uint32_t operator()(const uint8_t* p, size_t n) const {
        uint32_t c = 0xFFFFFFFFu;
        while (n >= 8) {
            const uint32_t lo = c ^ (uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24);
            const uint32_t hi = uint32_t(p[4]) | uint32_t(p[5]) << 8 | uint32_t(p[6]) << 16 | uint32_t(p[7]) << 24;
            c = t[7][lo & 0xFF] ^ t[6][(lo >> 8) & 0xFF] ^ t[5][(lo >> 16) & 0xFF] ^ t[4][lo >> 24] ^
                t[3][hi & 0xFF] ^ t[2][(hi >> 8) & 0xFF] ^ t[1][(hi >> 16) & 0xFF] ^ t[0][hi >> 24];
            p += 8;
            n -= 8;
        }
        while (n--) c = (c >> 8) ^ t[0][(c ^ *p++) & 0xFF];
        return c ^ 0xFFFFFFFFu;
    }
};

const Crc8& crc8() {
    static const Crc8 c;
    return c;
}

uint32_t be32(const uint8_t* p) { return uint32_t(p[0]) << 24 | uint32_t(p[1]) << 16 | uint32_t(p[2]) << 8 | p[3]; }

}  // namespace

// The file as PIL's PngImagePlugin reads it: the chunks before the first IDAT are CRC-checked
// and parsed (IHDR, PLTE; any other type skipped; a repeated IHDR replaces the earlier one);
// the image data is the run of consecutive IDAT chunks from there, taken without their CRCs
// (PIL does not check them; the zlib stream's Adler-32 covers the data), the last one possibly
// cut short by the end of the file; nothing after the run is read.
PngFileInfo png_parse(const uint8_t* data, size_t size, std::vector<std::pair<size_t, size_t>>* idat) {
    static const uint8_t sig[8] = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1A, '\n'};
    require(data != nullptr && size >= 8 && std::memcmp(data, sig, 8) == 0, "not a PNG file (signature)");
    PngFileInfo info{};
    size_t at = 8;
    bool ihdr = false;
    if (idat) idat->clear();
    for (;;) {
        require(size - at >= 12, "truncated PNG file (no image data)");
        const uint32_t len = be32(data + at);
        const uint8_t* type = data + at + 4;
        const uint8_t* body = data + at + 8;
        if (std::memcmp(type, "IDAT", 4) == 0) break;
        require(len <= size - at - 12, "truncated PNG chunk");
        if (crc8()(type, size_t(len) + 4) != be32(body + len))
            fail(AEISU_ERR_INVALID_ARG, std::string("broken PNG file: CRC mismatch in chunk ") +
                                            std::string(reinterpret_cast<const char*>(type), 4));
        if (std::memcmp(type, "IHDR", 4) == 0) {
            require(len == 13, "bad IHDR chunk");
            ihdr = true;
            info.w = int(be32(body));
            info.h = int(be32(body + 4));
            info.depth = body[8];
            info.color = body[9];
            info.interlace = body[12];
            require(info.w > 0 && info.h > 0 && be32(body) < (1u << 30) && be32(body + 4) < (1u << 30),
                    "bad PNG image size");
            require(body[10] == 0 && body[11] == 0, "unknown PNG compression or filter method");
        } else if (std::memcmp(type, "PLTE", 4) == 0) {
            info.npal = int(len / 3);   // a partial last entry is ignored
            std::memcpy(info.palette, body, std::min<size_t>(len / 3 * 3, sizeof(info.palette)));
        } else if (std::memcmp(type, "IEND", 4) == 0) {
            fail(AEISU_ERR_INVALID_ARG, "PNG file has no image data");
        }
        at += size_t(len) + 12;
    }
    require(ihdr, "IDAT before IHDR");
    while (size - at >= 8 && std::memcmp(data + at + 4, "IDAT", 4) == 0) {
        const size_t len = be32(data + at);
        const size_t take = std::min(len, size - at - 8);
        if (idat && take) idat->emplace_back(at + 8, take);
        info.idat_bytes += take;
        if (len + 12 > size - at) break;
        at += len + 12;
    }
    require(info.idat_bytes > 0, "PNG file has no image data");
    return info;
}

void png_check_supported(const PngFileInfo& info) {
    if (!(info.color == 0 || info.color == 2 || info.color == 3 || info.color == 4 || info.color == 6))
        fail(AEISU_ERR_INVALID_ARG, "bad PNG colour type " + std::to_string(info.color));
    if (info.depth != 8)
        fail(AEISU_ERR_UNSUPPORTED, "GPU PNG decode takes 8-bit samples only (bit depth " + std::to_string(info.depth) + ")");
    if (info.interlace != 0) fail(AEISU_ERR_UNSUPPORTED, "GPU PNG decode takes non-interlaced files only");
    if (info.color == 3) {
        // without a PLTE chunk every index reads as black, as PIL (12.x) decodes such a file
        require(info.npal <= 256, "invalid palette size");
    }
}

namespace {

// Device buffers kept between calls, per device: grow-only, and a call holds the device's lock
// from its first upload to its final synchronize, so concurrent calls on one device take turns.
// Like the tensor-map cache of the no-allocation entry point, they do not survive a reset of the
// device.
struct DecodeCache {
    enum { kIn, kFiles, kPal, kScratch, kStatus, kOut, kCount };
    std::mutex m;
    void* p[kCount] = {};
    size_t cap[kCount] = {};
    void* host = nullptr;   // page-locked staging of the zlib streams
    size_t host_cap = 0;
    uint8_t* get_host(size_t bytes) {
        if (host_cap < bytes) {
            if (host) cudaFreeHost(host);
            host = nullptr;
            host_cap = 0;
            const size_t want = bytes + bytes / 4;
            AEISU_CUDA(cudaHostAlloc(&host, want, cudaHostAllocDefault));
            host_cap = want;
        }
        return static_cast<uint8_t*>(host);
    }
    void* get(int k, size_t bytes) {
        if (cap[k] < bytes) {
            if (p[k]) cudaFree(p[k]);
            p[k] = nullptr;
            cap[k] = 0;
            const size_t want = bytes + bytes / 4;
            AEISU_CUDA(cudaMalloc(&p[k], want));
            cap[k] = want;
        }
        return p[k];
    }
};
constexpr int kMaxDecodeDevices = 64;

DecodeCache& decode_cache(int device) {
    static DecodeCache caches[kMaxDecodeDevices];
    return caches[device];
}

}  // namespace

void png_decode(const uint8_t* data, const uint64_t* offsets, const uint64_t* sizes, int n, int h, int w,
                bool host_out, int device, uint8_t* out, cudaStream_t stream) {
    require(data && offsets && sizes && out && n >= 1 && h >= 1 && w >= 1, "bad PNG decode arguments");
    require((unsigned long long)w * 4 + 1 < (1ull << 31), "PNG image too wide");
    require(device >= 0 && device < kMaxDecodeDevices, "bad device index");
    int prev = -1;
    AEISU_CUDA(cudaGetDevice(&prev));
    AEISU_CUDA(cudaSetDevice(device));
    struct Restore { int d; ~Restore() { if (d >= 0) cudaSetDevice(d); } } restore{prev};
    // host: parse and check every file; the zlib streams (without their 2-byte headers) are
    // gathered straight from the files into page-locked staging, each 16-byte aligned
    std::vector<DecFile> files(n);
    std::vector<std::vector<std::pair<size_t, size_t>>> idat(n);
    std::vector<uint8_t> pal;
    unsigned long long out_off = 0, in_off = 0;
    for (int i = 0; i < n; ++i) {
        const uint8_t* file = data + offsets[i];
        const PngFileInfo info = png_parse(file, size_t(sizes[i]), &idat[i]);
        png_check_supported(info);
        if (info.h != h || info.w != w)
            fail(AEISU_ERR_INVALID_ARG, "PNG file " + std::to_string(i) + " is " + std::to_string(info.w) + "x" +
                                            std::to_string(info.h) + ", the batch is " + std::to_string(w) + "x" +
                                            std::to_string(h));
        // zlib header (RFC 1950): deflate, window <= 32 KiB, no preset dictionary, check bits
        require(info.idat_bytes >= 6, "PNG image data too short");
        uint8_t head[2];
        for (int k = 0, r = 0, at = 0; k < 2; ++k) {   // the stream's first two bytes, across chunks
            while (size_t(at) >= idat[i][r].second) at -= int(idat[i][r++].second);
            head[k] = file[idat[i][r].first + at++];
        }
        const uint8_t cmf = head[0], flg = head[1];
        require((cmf & 15) == 8 && (cmf >> 4) <= 7 && ((cmf << 8) | flg) % 31 == 0 && !(flg & 0x20),
                "bad zlib header in PNG image data");
        DecFile& fd = files[i];
        fd.color = info.color;
        fd.bpp = info.color == 2 ? 3 : info.color == 6 ? 4 : info.color == 4 ? 2 : 1;
        fd.npal = info.color == 3 ? info.npal : 0;
        fd.pal_off = int(pal.size());
        if (fd.npal) pal.insert(pal.end(), info.palette, info.palette + 3 * fd.npal);
        fd.in_off = in_off;
        fd.in_len = info.idat_bytes - 2;
        in_off += (fd.in_len + 15) / 16 * 16;
        require((unsigned long long)h * (1ull + (unsigned long long)w * fd.bpp) < (1ull << 32), "PNG image too large");
        fd.out_off = out_off;
        out_off += ((unsigned long long)h * (1ull + (unsigned long long)w * fd.bpp) + 15) / 16 * 16;
    }
    const size_t in_bytes = size_t(in_off) + 16;   // + zero words the bit reader may load past an end
    if (pal.empty()) pal.push_back(0);
    DecGeom g{n, h, w, (unsigned long long)h * w * 3};
    DecodeCache& cache = decode_cache(device);
    std::lock_guard<std::mutex> lock(cache.m);
    uint8_t* staged = cache.get_host(in_bytes);
    for (int i = 0; i < n; ++i) {
        uint8_t* dst = staged + files[i].in_off;
        size_t skip = 2;   // the zlib header, checked above
        for (const auto& r : idat[i]) {
            if (skip >= r.second) {
                skip -= r.second;
                continue;
            }
            std::memcpy(dst, data + offsets[i] + r.first + skip, r.second - skip);
            dst += r.second - skip;
            skip = 0;
        }
        const uint8_t* end = staged + (i + 1 < n ? files[i + 1].in_off : in_bytes);
        std::memset(dst, 0, size_t(end - dst));
    }
    // once work is queued, the buffers stay locked until it is done, errors included
    struct Drain {
        cudaStream_t s;
        bool armed = false;
        ~Drain() { if (armed) cudaStreamSynchronize(s); }
    } drain{stream};
    void* d_in = cache.get(DecodeCache::kIn, in_bytes);
    void* d_files = cache.get(DecodeCache::kFiles, sizeof(DecFile) * n);
    void* d_pal = cache.get(DecodeCache::kPal, pal.size());
    // + slack: the unfilter stages whole aligned words and chunks past a row's end
    void* d_scratch = cache.get(DecodeCache::kScratch, out_off + 256);
    void* d_status = cache.get(DecodeCache::kStatus, sizeof(DecStatus) * n);
    uint8_t* dev_out = host_out ? static_cast<uint8_t*>(cache.get(DecodeCache::kOut, g.out_stride * n)) : out;
    drain.armed = true;
    AEISU_CUDA(cudaMemcpyAsync(d_in, staged, in_bytes, cudaMemcpyHostToDevice, stream));
    AEISU_CUDA(cudaMemcpyAsync(d_files, files.data(), sizeof(DecFile) * n, cudaMemcpyHostToDevice, stream));
    AEISU_CUDA(cudaMemcpyAsync(d_pal, pal.data(), pal.size(), cudaMemcpyHostToDevice, stream));
    AEISU_CUDA(cudaMemsetAsync(d_status, 0, sizeof(DecStatus) * n, stream));
    AEISU_CUDA(cudaFuncSetAttribute(k_png_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecodeSmem));
    k_png_decode<<<n, 64, kDecodeSmem, stream>>>(static_cast<const uint8_t*>(d_in), static_cast<const DecFile*>(d_files),
                                                 static_cast<uint8_t*>(d_scratch), static_cast<const uint8_t*>(d_pal), g,
                                                 dev_out, static_cast<DecStatus*>(d_status));
    AEISU_CUDA(cudaGetLastError());
    std::vector<DecStatus> st(n);
    AEISU_CUDA(cudaMemcpyAsync(st.data(), d_status, sizeof(DecStatus) * n, cudaMemcpyDeviceToHost, stream));
    if (host_out)
        AEISU_CUDA(cudaMemcpyAsync(out, dev_out, g.out_stride * n, cudaMemcpyDeviceToHost, stream));
    AEISU_CUDA(cudaStreamSynchronize(stream));
    drain.armed = false;
    static const char* what[] = {"", "bad deflate block", "bad Huffman code", "distance too far back",
                                 "more image data than the image holds", "truncated image data",
                                 "less image data than the image needs", "Adler-32 mismatch", "bad scanline filter type",
                                 "bad palette index", "decode wait limit reached"};
    for (int i = 0; i < n; ++i)
        if (st[i].error != kDecOk)
            fail(AEISU_ERR_INVALID_ARG, "PNG file " + std::to_string(i) + ": " +
                                            (st[i].error > 0 && st[i].error <= 10 ? what[st[i].error] : "decode error"));
}

}  // namespace aeisu
