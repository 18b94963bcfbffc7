// Baseline JPEG decoding behind pdefa_image_load (imageloader/src/jpeg/*.cpp).
//
// Sequential-DCT, Huffman-coded, 8-bit JPEG as ITU-T T.81 describes it, with
// the reference decoder's observable behaviour kept wherever it differs from
// the standard, because the pixels must match the reference's byte for byte:
//   * only the first scan is decoded, always with the interleaved MCU layout
//     (imageloader/src/jpeg/jpeg_decoder.cpp:96-151);
//   * the coefficient at zig-zag position i is multiplied by the quantiser at
//     NATURAL position i and truncated to int16 (jpeg_idct.cpp:13-18, tables
//     stored in natural order by jpeg_markers.cpp:96-97);
//   * a block without AC terms is filled with clamp(((dc*q0 + 4) >> 3) + 128)
//     (jpeg_decoder.cpp:119-123), which equals the IDCT's own result;
//   * the IDCT is the Chen-Wang integer 8x8 IDCT (the fixed-point form
//     published with the ISO MPEG-2 reference decoder: 11-bit constants
//     W_k = round(2048*sqrt(2)*cos(k*pi/16)), 8-bit row and 14-bit column
//     output shifts) (jpeg_idct.cpp:31-117);
//   * chroma (and the padded luma plane) is resampled by nearest index
//     s = x * plane_width / image_width over the MCU-padded plane
//     (jpeg_color.cpp:18-70), then converted with the 16-bit fixed-point
//     BT.601 full-range factors 1.402, 0.34414, 0.71414, 1.772;
//   * the bit reader un-stuffs 0xFF00, and after any other marker (or the end
//     of the data) supplies zero bits (jpeg_huffman.cpp:9-44).
// The Huffman decoder adds a 9-bit lookup in front of the canonical
// length-by-length search; the lookup returns exactly what the search would.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "image_io.h"

namespace pb {
namespace {

// Natural (row-major) index of zig-zag position i (T.81 Figure A.6).
constexpr uint8_t kZigzag[64] = {
    0,  1,  8,  16, 9,  2,  3,  10, 17, 24, 32, 25, 18, 11, 4,  5,
    12, 19, 26, 33, 40, 48, 41, 34, 27, 20, 13, 6,  7,  14, 21, 28,
    35, 42, 49, 56, 57, 50, 43, 36, 29, 22, 15, 23, 30, 37, 44, 51,
    58, 59, 52, 45, 38, 31, 39, 46, 53, 60, 61, 54, 47, 55, 62, 63};

struct JpegError {
    const char* what;
};
[[noreturn]] void fail(const char* m) { throw JpegError{m}; }

inline uint8_t sat8(int v) { return (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v)); }
inline int be16(const uint8_t* p) { return (p[0] << 8) | p[1]; }

// ---------------------------------------------------------------- Huffman
constexpr int kLookBits = 9;

struct HuffCode {
    uint8_t count[17] = {};      // codes of each length 1..16
    uint8_t sym[256] = {};
    int first[17] = {};          // first code value of each length
    int last[17] = {};           // last code value, -1 when the length has none
    int base[17] = {};           // index into sym of the first code of each length
    int nsym = 0;
    bool defined = false;
    uint16_t fast[1 << kLookBits] = {};   // (length << 8 | symbol), 0 = not resolved

    // Canonical code assignment (T.81 Annex C) with the reference's
    // bookkeeping: a length without codes gets last = -1 and keeps its other
    // fields (jpeg_markers.cpp:27-49).
    void assign() {
        int code = 0, k = 0;
        for (int len = 1; len <= 16; ++len) {
            if (count[len]) {
                base[len] = k;
                first[len] = code;
                code += count[len];
                k += count[len];
                last[len] = code - 1;
            } else {
                last[len] = -1;
            }
            code <<= 1;
        }
        nsym = k;
        defined = true;
        for (int p = 0; p < (1 << kLookBits); ++p) {
            fast[p] = 0;
            for (int len = 1; len <= kLookBits; ++len) {
                const int c = p >> (kLookBits - len);
                if (last[len] >= 0 && c <= last[len]) {
                    const int idx = base[len] + c - first[len];
                    if (idx >= 0 && idx < nsym) fast[p] = (uint16_t)(len << 8 | sym[idx]);
                    break;   // a bad index is left to the slow path, which reports it
                }
            }
        }
    }
};

// Entropy-coded segment reader. Bytes are taken in order with 0xFF00 read as
// 0xFF; at any other marker, or past the end, the stream continues with zero
// bits until the next restart. Reading ahead never crosses a marker, so the
// byte position at a restart search is equivalent to a bit-exact reader's.
class Bits {
public:
    Bits(const uint8_t* d, size_t n, size_t pos) : d_(d), n_(n), pos_(pos) {}

    uint32_t get(int n) {
        if (nbits_ < n) refill();
        nbits_ -= n;
        return (uint32_t)(acc_ >> nbits_) & ((1u << n) - 1u);
    }
    uint32_t peek(int n) {
        if (nbits_ < n) refill();
        return (uint32_t)(acc_ >> (nbits_ - n)) & ((1u << n) - 1u);
    }
    void skip(int n) { nbits_ -= n; }

    int decode(const HuffCode& h) {
        const uint16_t e = h.fast[peek(kLookBits)];
        if (e) {
            skip(e >> 8);
            return e & 0xFF;
        }
        int code = 0;
        for (int len = 1; len <= 16; ++len) {
            code = (code << 1) | (int)get(1);
            if (h.last[len] >= 0 && code <= h.last[len]) {
                const int idx = h.base[len] + code - h.first[len];
                if (idx < 0 || idx >= h.nsym) fail("jpeg: Huffman symbol index out of range");
                return h.sym[idx];
            }
        }
        fail("jpeg: invalid Huffman code");
    }

    // s magnitude bits -> signed value (T.81 F.2.2.1 EXTEND).
    int receive(int s) {
        if (s == 0) return 0;
        const int v = (int)get(s);
        return v < (1 << (s - 1)) ? v - (1 << s) + 1 : v;
    }

    // Drops buffered bits and moves past the next RSTn; false when another
    // marker or the end of the data comes first.
    bool restart() {
        acc_ = 0;
        nbits_ = 0;
        at_marker_ = false;
        while (pos_ + 1 < n_) {
            if (d_[pos_] != 0xFF) { ++pos_; continue; }
            const uint8_t m = d_[pos_ + 1];
            if (m >= 0xD0 && m <= 0xD7) { pos_ += 2; return true; }
            if (m != 0x00) return false;
            pos_ += 2;
        }
        return false;
    }

private:
    void refill() {
        while (nbits_ <= 56) {
            uint32_t b = 0;
            if (!at_marker_ && pos_ < n_) {
                b = d_[pos_];
                if (b != 0xFF) {
                    ++pos_;
                } else if (pos_ + 1 < n_ && d_[pos_ + 1] == 0x00) {
                    pos_ += 2;
                } else {
                    at_marker_ = true;
                    b = 0;
                }
            }
            acc_ = (acc_ << 8) | b;
            nbits_ += 8;
        }
    }

    const uint8_t* d_;
    size_t n_, pos_;
    uint64_t acc_ = 0;
    int nbits_ = 0;
    bool at_marker_ = false;
};

// ---------------------------------------------------------------- IDCT
// One 8-point pass of the Chen-Wang butterfly. kCol selects the column form:
// inputs scaled by 2^8 instead of 2^11, odd/even products rounded by >>3, and
// a 14-bit output shift with the +128 level shift and clamp applied by the
// caller. Integer evaluation order does not change the result.
template <bool kCol>
inline void chen_wang_8(const int* c, int step, int* y) {
    constexpr int W1 = 2841, W2 = 2676, W3 = 2408, W5 = 1609, W6 = 1108, W7 = 565;
    constexpr int kIn = kCol ? 8 : 11;
    const int c0 = c[0], c1 = c[step], c2 = c[2 * step], c3 = c[3 * step];
    const int c4 = c[4 * step], c5 = c[5 * step], c6 = c[6 * step], c7 = c[7 * step];
    auto r = [](int v) { return kCol ? (v + 4) >> 3 : v; };   // rounded product scale
    const int t17 = W7 * (c1 + c7), t53 = W3 * (c5 + c3), t26 = W6 * (c2 + c6);
    const int o1 = r(t17 + (W1 - W7) * c1), o7 = r(t17 - (W1 + W7) * c7);
    const int o5 = r(t53 - (W3 - W5) * c5), o3 = r(t53 - (W3 + W5) * c3);
    const int e2 = r(t26 + (W2 - W6) * c2), e6 = r(t26 - (W2 + W6) * c6);
    const int dc = c0 * (1 << kIn) + (kCol ? 8192 : 128);
    const int e0 = dc + c4 * (1 << kIn), e1 = dc - c4 * (1 << kIn);
    const int a = o1 + o5, b = o1 - o5, cc = o7 + o3, d = o7 - o3;
    const int f0 = e0 + e2, f3 = e0 - e2, f1 = e1 + e6, f2 = e1 - e6;
    const int g = (181 * (b + d) + 128) >> 8, h = (181 * (b - d) + 128) >> 8;
    constexpr int kOut = kCol ? 14 : 8;
    y[0] = (f0 + a) >> kOut;
    y[1] = (f1 + g) >> kOut;
    y[2] = (f2 + h) >> kOut;
    y[3] = (f3 + cc) >> kOut;
    y[4] = (f3 - cc) >> kOut;
    y[5] = (f2 - h) >> kOut;
    y[6] = (f1 - g) >> kOut;
    y[7] = (f0 - a) >> kOut;
}

// Dequantised natural-order coefficients -> 8x8 samples (stride `ld`).
void idct_block(const int16_t* coef, uint8_t* out, int ld) {
    int t[64];
    for (int i = 0; i < 8; ++i) {
        int row[8];
        for (int k = 0; k < 8; ++k) row[k] = coef[i * 8 + k];
        chen_wang_8<false>(row, 1, t + i * 8);
    }
    for (int x = 0; x < 8; ++x) {
        int col[8];
        chen_wang_8<true>(t + x, 8, col);
        for (int yy = 0; yy < 8; ++yy) out[yy * ld + x] = sat8(col[yy] + 128);
    }
}

// ---------------------------------------------------------------- frame
struct Plane {
    int id = 0, h = 1, v = 1, tq = 0, td = 0, ta = 0, pred = 0;
    int w = 0, rows = 0;             // MCU-padded plane size in samples
    std::vector<uint8_t> px;
};

struct Frame {
    int width = 0, height = 0, ncomp = 0;
    int hmax = 1, vmax = 1, mcux = 0, mcuy = 0;
    Plane comp[4];
    uint16_t q[4][64] = {};          // natural order
    bool qset[4] = {};
    HuffCode dc[4], ac[4];
    int restart_interval = 0;
    int nscan = 0, scan[4] = {};
    size_t scan_start = 0;
};

// Marker walk up to the first SOS (jpeg_markers.cpp:55-205): DQT, SOF0, DHT,
// DRI and SOS are read, SOF2 is refused, every other segment is skipped.
void parse(const uint8_t* d, size_t n, Frame& f) {
    if (n < 4 || d[0] != 0xFF || d[1] != 0xD8) fail("jpeg: missing SOI");
    size_t p = 2;
    bool sof = false, sos = false;
    while (p + 1 < n) {
        if (d[p] != 0xFF) { ++p; continue; }
        uint8_t m = d[p + 1];
        p += 2;
        while (m == 0xFF && p < n) m = d[p++];
        if (m == 0xD8 || m == 0x01 || (m >= 0xD0 && m <= 0xD7)) continue;
        if (m == 0xD9) break;
        if (p + 1 >= n) fail("jpeg: truncated segment length");
        const size_t len = (size_t)be16(d + p);
        if (len < 2 || p + len > n) fail("jpeg: segment runs past the end of the data");
        const uint8_t* s = d + p + 2;
        const size_t sn = len - 2;
        if (m == 0xDB) {
            for (size_t o = 0; o < sn;) {
                const int pq = s[o] >> 4, tq = s[o] & 15;
                ++o;
                if (pq != 0) fail("jpeg: 16-bit quantisation tables are not supported");
                if (tq > 3) fail("jpeg: quantisation table id out of range");
                if (o + 64 > sn) fail("jpeg: truncated DQT");
                for (int i = 0; i < 64; ++i) f.q[tq][kZigzag[i]] = s[o + i];
                f.qset[tq] = true;
                o += 64;
            }
        } else if (m == 0xC0) {
            if (sn < 6) fail("jpeg: short SOF0");
            if (s[0] != 8) fail("jpeg: only 8-bit samples are supported");
            f.height = be16(s + 1);
            f.width = be16(s + 3);
            f.ncomp = s[5];
            if (f.ncomp < 1 || f.ncomp > 4) fail("jpeg: component count out of range");
            for (int c = 0, o = 6; c < f.ncomp; ++c, o += 3) {
                if ((size_t)o + 3 > sn) fail("jpeg: truncated SOF0");
                Plane& pl = f.comp[c];
                pl.id = s[o];
                pl.h = s[o + 1] >> 4;
                pl.v = s[o + 1] & 15;
                pl.tq = s[o + 2];
                if (pl.h < 1 || pl.h > 4 || pl.v < 1 || pl.v > 4) fail("jpeg: sampling factor out of range");
            }
            f.hmax = f.vmax = 1;
            for (int c = 0; c < f.ncomp; ++c) {
                if (f.comp[c].h > f.hmax) f.hmax = f.comp[c].h;
                if (f.comp[c].v > f.vmax) f.vmax = f.comp[c].v;
            }
            f.mcux = (f.width + 8 * f.hmax - 1) / (8 * f.hmax);
            f.mcuy = (f.height + 8 * f.vmax - 1) / (8 * f.vmax);
            for (int c = 0; c < f.ncomp; ++c) {
                Plane& pl = f.comp[c];
                pl.w = f.mcux * pl.h * 8;
                pl.rows = f.mcuy * pl.v * 8;
                pl.px.assign((size_t)pl.w * pl.rows, 0);
            }
            sof = true;
        } else if (m == 0xC2) {
            fail("jpeg: progressive JPEG is not supported (baseline only)");
        } else if (m == 0xC4) {
            for (size_t o = 0; o < sn;) {
                const int tc = s[o] >> 4, th = s[o] & 15;
                ++o;
                if (tc > 1 || th > 3) fail("jpeg: DHT table class or id out of range");
                if (o + 16 > sn) fail("jpeg: short DHT");
                HuffCode& h = tc == 0 ? f.dc[th] : f.ac[th];
                int total = 0;
                for (int i = 1; i <= 16; ++i) total += (h.count[i] = s[o + i - 1]);
                o += 16;
                if (total > 256 || o + (size_t)total > sn) fail("jpeg: DHT symbol list runs past the segment");
                std::memcpy(h.sym, s + o, (size_t)total);
                o += (size_t)total;
                h.assign();
            }
        } else if (m == 0xDD) {
            if (sn < 2) fail("jpeg: short DRI");
            f.restart_interval = be16(s);
        } else if (m == 0xDA) {
            if (!sof) fail("jpeg: SOS before SOF");
            if (sn < 4) fail("jpeg: short SOS");
            f.nscan = s[0];
            if (f.nscan < 1 || f.nscan > f.ncomp) fail("jpeg: SOS component count out of range");
            size_t o = 1;
            for (int i = 0; i < f.nscan; ++i, o += 2) {
                if (o + 2 > sn) fail("jpeg: truncated SOS");
                int ci = -1;
                for (int c = 0; c < f.ncomp && ci < 0; ++c)
                    if (f.comp[c].id == s[o]) ci = c;
                if (ci < 0) fail("jpeg: SOS names an unknown component");
                f.scan[i] = ci;
                f.comp[ci].td = s[o + 1] >> 4;
                f.comp[ci].ta = s[o + 1] & 15;
            }
            if (o + 3 > sn) fail("jpeg: truncated SOS");
            if (s[o] != 0 || s[o + 1] != 63 || s[o + 2] != 0) fail("jpeg: not a baseline scan (progressive?)");
            f.scan_start = p + len;
            sos = true;
            break;
        }
        p += len;
    }
    if (!sof) fail("jpeg: no SOF0 segment");
    if (!sos) fail("jpeg: no SOS segment");
}

// One 8x8 block: Huffman-decode the 64 zig-zag coefficients, then write its
// samples at (bx, by) of the plane.
void decode_block(Bits& br, Plane& pl, const HuffCode& hd, const HuffCode& ha, const uint16_t* q,
                  int bx, int by) {
    int16_t zz[64];
    std::memset(zz, 0, sizeof(zz));
    const int t = br.decode(hd);
    if (t > 15) fail("jpeg: DC magnitude category out of range");
    pl.pred += br.receive(t);
    zz[0] = (int16_t)pl.pred;
    bool any_ac = false;
    for (int k = 1; k < 64;) {
        const int rs = br.decode(ha);
        const int run = rs >> 4, size = rs & 15;
        if (size == 0) {
            if (run != 15) break;    // EOB
            k += 16;                 // ZRL
            continue;
        }
        k += run;
        if (k >= 64) fail("jpeg: AC run past the end of the block");
        zz[k++] = (int16_t)br.receive(size);
        any_ac = true;
    }
    uint8_t* dst = pl.px.data() + (size_t)by * pl.w + bx;
    if (!any_ac) {
        const uint8_t v = sat8(((zz[0] * q[0] + 4) >> 3) + 128);
        for (int r = 0; r < 8; ++r) std::memset(dst + (size_t)r * pl.w, v, 8);
        return;
    }
    int16_t nat[64];
    for (int i = 0; i < 64; ++i) nat[kZigzag[i]] = (int16_t)(zz[i] * q[i]);
    idct_block(nat, dst, pl.w);
}

void decode_scan(const uint8_t* d, size_t n, Frame& f) {
    const HuffCode* hd[4];
    const HuffCode* ha[4];
    for (int s = 0; s < f.nscan; ++s) {
        const Plane& pl = f.comp[f.scan[s]];
        if (pl.td > 3 || pl.ta > 3 || !f.dc[pl.td].defined || !f.ac[pl.ta].defined)
            fail("jpeg: missing Huffman table");
        if (pl.tq > 3 || !f.qset[pl.tq]) fail("jpeg: missing quantisation table");
        hd[s] = &f.dc[pl.td];
        ha[s] = &f.ac[pl.ta];
    }
    Bits br(d, n, f.scan_start);
    const int total = f.mcux * f.mcuy;
    int since_restart = 0;
    for (int mcu = 0; mcu < total; ++mcu) {
        const int mx = mcu % f.mcux, my = mcu / f.mcux;
        for (int s = 0; s < f.nscan; ++s) {
            Plane& pl = f.comp[f.scan[s]];
            for (int vy = 0; vy < pl.v; ++vy)
                for (int hx = 0; hx < pl.h; ++hx)
                    decode_block(br, pl, *hd[s], *ha[s], f.q[pl.tq], (mx * pl.h + hx) * 8, (my * pl.v + vy) * 8);
        }
        if (f.restart_interval > 0 && ++since_restart == f.restart_interval && mcu + 1 < total) {
            if (!br.restart()) fail("jpeg: expected RST marker not found");
            for (int c = 0; c < f.ncomp; ++c) f.comp[c].pred = 0;
            since_restart = 0;
        }
    }
}

// Nearest-index resampling of each plane to the image size, then YCbCr -> RGB
// (one component: grey replicated into RGB).
void to_rgb(const Frame& f, uint8_t* out) {
    const int W = f.width, H = f.height;
    const int nc = f.ncomp == 1 ? 1 : 3;
    if (f.ncomp == 2) fail("jpeg: colour images need 3 or more components");
    std::vector<int> sx((size_t)nc * W);
    for (int c = 0; c < nc; ++c)
        for (int x = 0; x < W; ++x) {
            int v = (int)((int64_t)x * f.comp[c].w / W);
            sx[(size_t)c * W + x] = v < f.comp[c].w ? v : f.comp[c].w - 1;
        }
    for (int y = 0; y < H; ++y) {
        const uint8_t* row[3];
        for (int c = 0; c < nc; ++c) {
            int sy = (int)((int64_t)y * f.comp[c].rows / H);
            if (sy >= f.comp[c].rows) sy = f.comp[c].rows - 1;
            row[c] = f.comp[c].px.data() + (size_t)sy * f.comp[c].w;
        }
        uint8_t* o = out + (size_t)y * W * 3;
        if (nc == 1) {
            for (int x = 0; x < W; ++x) o[3 * x] = o[3 * x + 1] = o[3 * x + 2] = row[0][sx[x]];
            continue;
        }
        const int* sy0 = sx.data();
        const int* sy1 = sx.data() + W;
        const int* sy2 = sx.data() + 2 * (size_t)W;
        for (int x = 0; x < W; ++x) {
            const int Y = row[0][sy0[x]], cb = row[1][sy1[x]] - 128, cr = row[2][sy2[x]] - 128;
            o[3 * x + 0] = sat8(Y + ((91881 * cr) >> 16));
            o[3 * x + 1] = sat8(Y - ((22554 * cb + 46802 * cr) >> 16));
            o[3 * x + 2] = sat8(Y + ((116130 * cb) >> 16));
        }
    }
}

}  // namespace

bool decode_jpeg(const uint8_t* d, size_t n, DecodedImage& img, std::string& err) {
    try {
        if (n < 4 || d[0] != 0xFF || d[1] != 0xD8) fail("jpeg: bad signature (no SOI)");
        Frame f;
        parse(d, n, f);
        if (f.scan_start == 0 || f.scan_start >= n) fail("jpeg: no entropy-coded data");
        decode_scan(d, n, f);
        img.width = (uint32_t)f.width;
        img.height = (uint32_t)f.height;
        img.format = kFmtRGB8;
        img.pixels.assign((size_t)f.width * f.height * 3, 0);
        to_rgb(f, img.pixels.data());
        return true;
    } catch (const JpegError& e) {
        err = e.what;
        return false;
    }
}

}  // namespace pb
