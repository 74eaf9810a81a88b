// Deflate (RFC 1951) pieces of the PNG encoder that one thread runs per segment: length-limited
// Huffman code lengths, canonical codes, the run-length coding of the code lengths, the
// dynamic block header and the length / distance symbol tables of RFC 1951 3.2.5.  Host and
// device code (the host build is the CPU check of this logic against zlib); the match search,
// the bit emission and the PNG framing are in k_png.cu.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define DEFL_HD __host__ __device__ __forceinline__
#else
#define DEFL_HD inline
#endif

namespace aeisu {
namespace defl {

constexpr int kLit = 286;           // literal/length alphabet: bytes, end of block (256), lengths
constexpr int kDist = 30;           // distance alphabet
constexpr int kLens = kLit + kDist; // most code lengths a header sends
constexpr int kCl = 19;             // code-length alphabet
constexpr int kLitLimit = 15, kClLimit = 7;
constexpr int kMinMatch = 4, kMaxMatch = 258, kWindow = 32768;

DEFL_HD int ilog2(uint32_t v) {
    int e = 0;
    while (v >>= 1) ++e;
    return e;
}

// Length 3..258 -> symbol 257..285, extra bits and their value (RFC 1951 3.2.5): lengths
// 3-10 have symbols of their own, then each group of four symbols doubles the span, 258 is 285.
DEFL_HD int length_symbol(int len, int& nextra, int& extra) {
    if (len == kMaxMatch) return nextra = 0, extra = 0, 285;
    if (len < 11) return nextra = 0, extra = 0, 254 + len;
    const int x = len - 3, e = ilog2(uint32_t(x));
    nextra = e - 2;
    extra = x & ((1 << nextra) - 1);
    return 257 + 4 * (e - 1) + ((x >> (e - 2)) & 3);
}

// Distance 1..32768 -> symbol 0..29 with its extra bits (RFC 1951 3.2.5): 1-4 have symbols of
// their own, then each pair of symbols doubles the span.
DEFL_HD int distance_symbol(int dist, int& nextra, int& extra) {
    if (dist <= 4) return nextra = 0, extra = 0, dist - 1;
    const int x = dist - 1, e = ilog2(uint32_t(x));
    nextra = e - 1;
    extra = x & ((1 << nextra) - 1);
    return 2 * e + ((x >> (e - 1)) & 1);
}

// Order in which the code-length code lengths are sent (RFC 1951 3.2.7).
DEFL_HD int cl_order(int k) {
    constexpr int8_t o[kCl] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};
    return o[k];
}

// Scratch of the Huffman construction for an alphabet of up to n symbols.
struct HuffScratch {
    uint32_t* weight;   // [2n]
    uint16_t* parent;   // [2n]
    uint16_t* sorted;   // [n]: used symbols in ascending (frequency, symbol) order
};

// Code lengths <= limit for symbols sorted[0..m) with frequencies freq[] (all > 0, m >= 1):
// Huffman's construction with two queues (leaves in sorted order, merged nodes in creation
// order, both non-decreasing), then depths from the root down.  If the deepest leaf exceeds
// `limit`, every weight becomes (w >> 1) | 1 (same order, flatter distribution) and the code is
// rebuilt.  A single used symbol gets length 1 (one-bit code, the other code unused).
DEFL_HD void huffman_lengths(uint32_t* freq, int m, int limit, uint8_t* len, HuffScratch s) {
    if (m == 1) {
        len[s.sorted[0]] = 1;
        return;
    }
    for (int i = 0; i < m; ++i) s.weight[i] = freq[s.sorted[i]];
    for (;;) {
        int leaf = 0, node = m, next = m;
        auto take = [&]() {
            if (leaf < m && (node >= next || s.weight[leaf] <= s.weight[node])) return leaf++;
            return node++;
        };
        for (int k = 0; k < m - 1; ++k) {
            const int a = take(), b = take();
            s.weight[next] = s.weight[a] + s.weight[b];
            s.parent[a] = s.parent[b] = uint16_t(next);
            ++next;
        }
        // depth of every node: the root (last node) is 0, parents precede children going down
        const int root = 2 * m - 2;
        s.weight[root] = 0;   // reused as depth from here on
        int deepest = 0;
        for (int i = root - 1; i >= 0; --i) {
            s.weight[i] = s.weight[s.parent[i]] + 1;
            if (i < m && int(s.weight[i]) > deepest) deepest = int(s.weight[i]);
        }
        if (deepest <= limit) {
            for (int i = 0; i < m; ++i) len[s.sorted[i]] = uint8_t(s.weight[i]);
            return;
        }
        for (int i = 0; i < m; ++i) {   // flattened weights replace the frequencies
            freq[s.sorted[i]] = (freq[s.sorted[i]] >> 1) | 1u;
            s.weight[i] = freq[s.sorted[i]];
        }
    }
}

// Used symbols of freq[0..n) in ascending (frequency, symbol) order by insertion; returns m.
DEFL_HD int sort_used(const uint32_t* freq, int n, uint16_t* sorted) {
    int m = 0;
    for (int sym = 0; sym < n; ++sym) {
        if (!freq[sym]) continue;
        int j = m++;
        while (j > 0 && (freq[sorted[j - 1]] > freq[sym])) {
            sorted[j] = sorted[j - 1];
            --j;
        }
        sorted[j] = uint16_t(sym);
    }
    return m;
}

DEFL_HD uint32_t reverse_bits(uint32_t v, int n) {
    uint32_t r = 0;
    for (int i = 0; i < n; ++i) r |= ((v >> i) & 1u) << (n - 1 - i);
    return r;
}

// Canonical codes (RFC 1951 3.2.2) from code lengths, bit-reversed for LSB-first emission.
DEFL_HD void canonical_codes(const uint8_t* len, int n, uint16_t* code_rev) {
    uint16_t count[16] = {0}, next[16] = {0};
    for (int i = 0; i < n; ++i) count[len[i]]++;
    count[0] = 0;
    uint16_t c = 0;
    for (int b = 1; b < 16; ++b) {
        c = uint16_t((c + count[b - 1]) << 1);
        next[b] = c;
    }
    for (int i = 0; i < n; ++i)
        code_rev[i] = len[i] ? uint16_t(reverse_bits(next[len[i]]++, len[i])) : 0;
}

// Run-length coding of the header's code lengths (RFC 1951 3.2.7): symbols 0-15 literal
// lengths, 16 = repeat the previous length 3-6 times (2 extra bits), 17 = 3-10 zeros (3 bits),
// 18 = 11-138 zeros (7 bits).  Writes (symbol, extra) pairs; returns their count.
DEFL_HD int rle_lengths(const uint8_t* lens, int n, uint8_t* sym, uint8_t* extra) {
    int k = 0, i = 0;
    while (i < n) {
        const uint8_t v = lens[i];
        int run = 1;
        while (i + run < n && lens[i + run] == v) ++run;
        i += run;
        if (v == 0) {
            while (run >= 11) {
                const int r = run < 138 ? run : 138;
                sym[k] = 18, extra[k++] = uint8_t(r - 11);
                run -= r;
            }
            if (run >= 3) {
                sym[k] = 17, extra[k++] = uint8_t(run - 3);
                run = 0;
            }
            while (run-- > 0) sym[k] = 0, extra[k++] = 0;
        } else {
            sym[k] = v, extra[k++] = 0;
            --run;
            while (run >= 3) {
                const int r = run < 6 ? run : 6;
                sym[k] = 16, extra[k++] = uint8_t(r - 3);
                run -= r;
            }
            while (run-- > 0) sym[k] = v, extra[k++] = 0;
        }
    }
    return k;
}

DEFL_HD int extra_bits(int clsym) { return clsym == 16 ? 2 : clsym == 17 ? 3 : clsym == 18 ? 7 : 0; }

// Everything the block header needs, built by one thread from the symbol frequencies.
struct Header {
    uint8_t lit_len[kLit];
    uint16_t lit_code[kLit];
    uint8_t dist_len[kDist];
    uint16_t dist_code[kDist];
    uint8_t cl_len[kCl];
    uint16_t cl_code[kCl];
    uint8_t rle_sym[kLens];
    uint8_t rle_extra[kLens];
    int nlit, ndist;   // code lengths sent for each alphabet (HLIT + 257, HDIST + 1)
    int nrle;
    int hclen;         // code-length code lengths sent (4..19)
    int bits;          // header size in bits, BFINAL/BTYPE included
};

// freq[kLit] / dfreq[kDist] are the literal/length and distance histograms (freq[256] = 1 for
// the end of block); both may be flattened when a code has to be length-limited.
// s.sorted[0..m) must hold the m used literal/length symbols in ascending (frequency, symbol)
// order (sort_used, or a parallel ranking).  scratch: weight[2*kLit], parent[2*kLit],
// sorted[kLit].  A block without matches still sends two distance codes of length 1, a
// complete code that every inflater accepts.
DEFL_HD void build_header(uint32_t* freq, int m, uint32_t* dfreq, Header& h, HuffScratch s) {
    for (int i = 0; i < kLit; ++i) h.lit_len[i] = 0;
    huffman_lengths(freq, m, kLitLimit, h.lit_len, s);
    for (int i = 0; i < kDist; ++i) h.dist_len[i] = 0;
    const int md = sort_used(dfreq, kDist, s.sorted);
    if (md == 0) {
        h.dist_len[0] = h.dist_len[1] = 1;
    } else {
        huffman_lengths(dfreq, md, kLitLimit, h.dist_len, s);
        if (md == 1) h.dist_len[s.sorted[0] == 0 ? 1 : 0] = 1;   // complete the one-symbol code
    }
    canonical_codes(h.lit_len, kLit, h.lit_code);
    canonical_codes(h.dist_len, kDist, h.dist_code);
    h.nlit = kLit;
    while (h.nlit > 257 && h.lit_len[h.nlit - 1] == 0) --h.nlit;
    h.ndist = kDist;
    while (h.ndist > 1 && h.dist_len[h.ndist - 1] == 0) --h.ndist;
    uint8_t lens[kLens];
    for (int i = 0; i < h.nlit; ++i) lens[i] = h.lit_len[i];
    for (int i = 0; i < h.ndist; ++i) lens[h.nlit + i] = h.dist_len[i];
    h.nrle = rle_lengths(lens, h.nlit + h.ndist, h.rle_sym, h.rle_extra);
    uint32_t clf[kCl] = {0};
    for (int k = 0; k < h.nrle; ++k) clf[h.rle_sym[k]]++;
    for (int i = 0; i < kCl; ++i) h.cl_len[i] = 0;
    const int mc = sort_used(clf, kCl, s.sorted);
    huffman_lengths(clf, mc, kClLimit, h.cl_len, s);
    if (mc == 1) h.cl_len[s.sorted[0] == 0 ? 1 : 0] = 1;
    canonical_codes(h.cl_len, kCl, h.cl_code);
    h.hclen = kCl;
    while (h.hclen > 4 && h.cl_len[cl_order(h.hclen - 1)] == 0) --h.hclen;
    int bits = 3 + 5 + 5 + 4 + 3 * h.hclen;
    for (int k = 0; k < h.nrle; ++k) bits += h.cl_len[h.rle_sym[k]] + extra_bits(h.rle_sym[k]);
    h.bits = bits;
}

// Writes the header through put(value, nbits) (LSB-first fields, bit-reversed codes).
template <typename Put>
DEFL_HD void write_header(const Header& h, bool final, Put&& put) {
    put(final ? 1u : 0u, 1);
    put(2u, 2);                          // BTYPE = 10: dynamic Huffman codes
    put(uint32_t(h.nlit - 257), 5);      // HLIT
    put(uint32_t(h.ndist - 1), 5);       // HDIST
    put(uint32_t(h.hclen - 4), 4);       // HCLEN
    for (int k = 0; k < h.hclen; ++k) put(h.cl_len[cl_order(k)], 3);
    for (int k = 0; k < h.nrle; ++k) {
        const int s = h.rle_sym[k];
        put(h.cl_code[s], h.cl_len[s]);
        if (extra_bits(s)) put(h.rle_extra[k], extra_bits(s));
    }
}

// A parsed token: a literal byte (value < 65536) or a match, (length << 16) | (distance - 1).
DEFL_HD uint32_t match_token(int len, int dist) { return (uint32_t(len) << 16) | uint32_t(dist - 1); }

// Bits of one token under the block's codes.
DEFL_HD int token_bits(const Header& h, uint32_t tok) {
    if (tok < 65536u) return h.lit_len[tok];
    int ne, ev, de, dv;
    const int ls = length_symbol(int(tok >> 16), ne, ev);
    const int ds = distance_symbol(int(tok & 0xFFFF) + 1, de, dv);
    return h.lit_len[ls] + ne + h.dist_len[ds] + de;
}

// Emits one token through put(value, nbits).
template <typename Put>
DEFL_HD void put_token(const Header& h, uint32_t tok, Put&& put) {
    if (tok < 65536u) {
        put(h.lit_code[tok], h.lit_len[tok]);
        return;
    }
    int ne, ev, de, dv;
    const int ls = length_symbol(int(tok >> 16), ne, ev);
    const int ds = distance_symbol(int(tok & 0xFFFF) + 1, de, dv);
    put(h.lit_code[ls], h.lit_len[ls]);
    if (ne) put(uint32_t(ev), ne);
    put(h.dist_code[ds], h.dist_len[ds]);
    if (de) put(uint32_t(dv), de);
}

}  // namespace defl
}  // namespace aeisu
