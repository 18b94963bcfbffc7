// PNG decoding for pdefa_image_load (replaces imageloader/src/png/*.cpp, used by
// imageloader/src/loader.cpp for files that start with the PNG signature).
//
// Written from the PNG specification (ISO/IEC 15948): chunk walk with CRC checks,
// zlib inflate (the system zlib), the five row filters, sample unpacking for every
// bit depth, Adam7 de-interlacing. The decoded pixels follow the reference's
// conversions (imageloader/src/png/png_unpack.cpp), so both libraries return the
// same bytes for the same file:
//   gray (1-8 bit) -> GRAY8, 16-bit gray -> GRAY16 (big-endian bytes), gray + tRNS ->
//   RGBA8 (alpha 0 where the raw sample equals the tRNS gray); RGB -> RGB8, RGB + tRNS
//   -> RGBA8 except 8-bit non-interlaced RGB, which stays RGB8; palette -> RGB8 (RGBA8 with tRNS alpha); gray+alpha and RGBA -> RGBA8;
//   16-bit samples keep their high byte, sub-byte samples scale as (v*255 + max/2)/max.
#include <zlib.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "image_io.h"

namespace pb {

namespace {

uint32_t be32(const uint8_t* p) { return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3]; }

int channels_of(int color_type) {
    switch (color_type) {
        case 0: return 1;
        case 2: return 3;
        case 3: return 1;
        case 4: return 2;
        case 6: return 4;
    }
    return 0;
}

size_t row_bytes_of(uint32_t w, int ct, int bd) { return ((size_t)w * bd * channels_of(ct) + 7) / 8; }

uint8_t paeth(int a, int b, int c) {
    const int p = a + b - c;
    const int pa = p > a ? p - a : a - p, pb = p > b ? p - b : b - p, pc = p > c ? p - c : c - p;
    return (uint8_t)((pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c));
}

// Undo the row filters of one (sub)image: raw = h rows of (1 + rb) bytes; out = h * rb.
bool unfilter(const uint8_t* raw, uint32_t h, size_t rb, size_t bpp, std::vector<uint8_t>& out, std::string& err) {
    out.assign((size_t)h * rb, 0);
    for (uint32_t y = 0; y < h; ++y) {
        const uint8_t ft = raw[(size_t)y * (rb + 1)];
        const uint8_t* src = raw + (size_t)y * (rb + 1) + 1;
        uint8_t* cur = out.data() + (size_t)y * rb;
        const uint8_t* prev = y ? cur - rb : nullptr;
        for (size_t i = 0; i < rb; ++i) {
            const int a = i >= bpp ? cur[i - bpp] : 0;
            const int b = prev ? prev[i] : 0;
            const int c = (prev && i >= bpp) ? prev[i - bpp] : 0;
            switch (ft) {
                case 0: cur[i] = src[i]; break;
                case 1: cur[i] = (uint8_t)(src[i] + a); break;
                case 2: cur[i] = (uint8_t)(src[i] + b); break;
                case 3: cur[i] = (uint8_t)(src[i] + ((a + b) >> 1)); break;
                case 4: cur[i] = (uint8_t)(src[i] + paeth(a, b, c)); break;
                default: err = "png: unknown row filter"; return false;
            }
        }
    }
    return true;
}

uint16_t sample_at(const uint8_t* row, size_t k, int bd) {
    if (bd == 8) return row[k];
    if (bd == 16) return (uint16_t)(row[2 * k] << 8 | row[2 * k + 1]);
    const int per = 8 / bd;
    const int shift = 8 - bd * (int)(k % per + 1);
    return (uint16_t)((row[k / per] >> shift) & ((1 << bd) - 1));
}

uint8_t to8(uint16_t v, int bd) {
    if (bd == 8) return (uint8_t)v;
    if (bd == 16) return (uint8_t)(v >> 8);
    const int mx = (1 << bd) - 1;
    return (uint8_t)((v * 255 + mx / 2) / mx);
}

}  // namespace

bool decode_png(const uint8_t* d, size_t n, DecodedImage& img, std::string& err) {
    static const uint8_t kSig[8] = {0x89, 'P', 'N', 'G', 0x0D, 0x0A, 0x1A, 0x0A};
    if (n < 8 || std::memcmp(d, kSig, 8) != 0) { err = "png: bad signature"; return false; }
    uint32_t W = 0, H = 0;
    int bd = 0, ct = 0, interlace = 0;
    bool ihdr = false, iend = false, has_trns = false;
    std::vector<uint8_t> plte, trns, idat;
    for (size_t pos = 8; pos + 8 <= n && !iend;) {
        const uint32_t len = be32(d + pos);
        const uint8_t* type = d + pos + 4;
        if (len > n || pos + 12 + (size_t)len > n) { err = "png: chunk runs past the end of the file"; return false; }
        const uint8_t* data = type + 4;
        const uint32_t crc = (uint32_t)crc32(crc32(0L, Z_NULL, 0), type, len + 4);
        if (crc != be32(data + len)) { err = "png: chunk CRC mismatch"; return false; }
        if (!std::memcmp(type, "IHDR", 4)) {
            if (len != 13) { err = "png: IHDR length must be 13"; return false; }
            W = be32(data); H = be32(data + 4);
            bd = data[8]; ct = data[9];
            if (data[10] != 0 || data[11] != 0) { err = "png: unsupported compression or filter method"; return false; }
            interlace = data[12];
            ihdr = true;
        } else if (!std::memcmp(type, "PLTE", 4)) {
            if (len % 3 || len > 768) { err = "png: bad PLTE length"; return false; }
            plte.assign(data, data + len);
        } else if (!std::memcmp(type, "tRNS", 4)) {
            trns.assign(data, data + len);
            has_trns = true;
        } else if (!std::memcmp(type, "IDAT", 4)) {
            idat.insert(idat.end(), data, data + len);
        } else if (!std::memcmp(type, "IEND", 4)) {
            iend = true;
        }
        pos += 12 + (size_t)len;
    }
    if (!ihdr) { err = "png: no IHDR"; return false; }
    if (idat.empty()) { err = "png: no IDAT data"; return false; }
    if (!iend) { err = "png: no IEND"; return false; }
    if (interlace > 1) { err = "png: bad interlace method"; return false; }
    if (W == 0 || H == 0) { err = "png: zero size"; return false; }
    const bool ok_depth = (ct == 0 && (bd == 1 || bd == 2 || bd == 4 || bd == 8 || bd == 16)) ||
                          (ct == 3 && (bd == 1 || bd == 2 || bd == 4 || bd == 8)) ||
                          ((ct == 2 || ct == 4 || ct == 6) && (bd == 8 || bd == 16));
    if (!channels_of(ct) || !ok_depth) { err = "png: unsupported colour type / bit depth"; return false; }
    if (ct == 3 && plte.empty()) { err = "png: palette image without PLTE"; return false; }
    const int ch = channels_of(ct);
    const size_t bpp = std::max<size_t>(1, ((size_t)bd * ch + 7) / 8);

    // passes: (x0, y0, dx, dy); one full pass without interlace
    static const int kAdam7[7][4] = {{0, 0, 8, 8}, {4, 0, 8, 8}, {0, 4, 4, 8}, {2, 0, 4, 4},
                                     {0, 2, 2, 4}, {1, 0, 2, 2}, {0, 1, 1, 2}};
    const int npass = interlace ? 7 : 1;
    size_t total_raw = 0;
    std::vector<uint32_t> pw(npass), ph(npass);
    for (int q = 0; q < npass; ++q) {
        const int x0 = interlace ? kAdam7[q][0] : 0, y0 = interlace ? kAdam7[q][1] : 0;
        const int dx = interlace ? kAdam7[q][2] : 1, dy = interlace ? kAdam7[q][3] : 1;
        pw[q] = (uint32_t)x0 < W ? (W - x0 + dx - 1) / dx : 0;
        ph[q] = (uint32_t)y0 < H ? (H - y0 + dy - 1) / dy : 0;
        if (pw[q] && ph[q]) total_raw += (row_bytes_of(pw[q], ct, bd) + 1) * ph[q];
    }
    std::vector<uint8_t> raw(total_raw);
    z_stream zs{};
    if (inflateInit(&zs) != Z_OK) { err = "png: zlib init failed"; return false; }
    zs.next_in = idat.data();
    zs.avail_in = (uInt)idat.size();
    zs.next_out = raw.data();
    zs.avail_out = (uInt)raw.size();
    const int zr = inflate(&zs, Z_FINISH);
    const size_t got = raw.size() - zs.avail_out;
    inflateEnd(&zs);
    if ((zr != Z_STREAM_END && zr != Z_BUF_ERROR && zr != Z_OK) || got < total_raw) {
        err = "png: compressed image data is truncated or corrupt";
        return false;
    }

    std::vector<uint8_t> rows;
    if (!interlace && bd == 8 && (ct == 2 || ct == 6)) {
        // 8-bit RGB / RGBA without interlacing: the unfiltered rows are the pixels (the
        // reference takes this path before looking at tRNS, so RGB + tRNS stays RGB8)
        if (!unfilter(raw.data(), H, row_bytes_of(W, ct, bd), bpp, rows, err)) return false;
        img.width = W;
        img.height = H;
        img.format = ct == 2 ? kFmtRGB8 : kFmtRGBA8;
        img.pixels = std::move(rows);
        return true;
    }
    std::vector<uint16_t> canvas((size_t)W * H * ch, 0);
    size_t off = 0;
    for (int q = 0; q < npass; ++q) {
        if (!pw[q] || !ph[q]) continue;
        const int x0 = interlace ? kAdam7[q][0] : 0, y0 = interlace ? kAdam7[q][1] : 0;
        const int dx = interlace ? kAdam7[q][2] : 1, dy = interlace ? kAdam7[q][3] : 1;
        const size_t rb = row_bytes_of(pw[q], ct, bd);
        if (!unfilter(raw.data() + off, ph[q], rb, bpp, rows, err)) return false;
        off += (rb + 1) * ph[q];
        for (uint32_t y = 0; y < ph[q]; ++y) {
            const uint8_t* row = rows.data() + (size_t)y * rb;
            const size_t cy = y0 + (size_t)y * dy;
            for (uint32_t x = 0; x < pw[q]; ++x) {
                const size_t cx = x0 + (size_t)x * dx;
                for (int c = 0; c < ch; ++c) canvas[(cy * W + cx) * ch + c] = sample_at(row, (size_t)x * ch + c, bd);
            }
        }
    }

    const size_t total = (size_t)W * H;
    img.width = W;
    img.height = H;
    uint16_t tg = 0, tr = 0, tgr = 0, tb = 0;
    if (has_trns && ct == 0) {
        if (trns.size() < 2) { err = "png: short tRNS for a gray image"; return false; }
        tg = (uint16_t)(trns[0] << 8 | trns[1]);
    } else if (has_trns && ct == 2) {
        if (trns.size() < 6) { err = "png: short tRNS for an RGB image"; return false; }
        tr = (uint16_t)(trns[0] << 8 | trns[1]);
        tgr = (uint16_t)(trns[2] << 8 | trns[3]);
        tb = (uint16_t)(trns[4] << 8 | trns[5]);
    }
    auto out4 = [&](size_t i, uint8_t r, uint8_t g, uint8_t b, uint8_t a) {
        img.pixels[i * 4] = r; img.pixels[i * 4 + 1] = g; img.pixels[i * 4 + 2] = b; img.pixels[i * 4 + 3] = a;
    };
    if (ct == 0) {
        if (has_trns) {
            img.format = kFmtRGBA8;
            img.pixels.assign(total * 4, 0);
            for (size_t i = 0; i < total; ++i) {
                const uint8_t v = to8(canvas[i], bd);
                out4(i, v, v, v, canvas[i] == tg ? 0 : 255);
            }
        } else if (bd == 16) {
            img.format = kFmtGRAY16;
            img.pixels.assign(total * 2, 0);
            for (size_t i = 0; i < total; ++i) {
                img.pixels[2 * i] = (uint8_t)(canvas[i] >> 8);
                img.pixels[2 * i + 1] = (uint8_t)(canvas[i] & 0xFF);
            }
        } else {
            img.format = kFmtGRAY8;
            img.pixels.assign(total, 0);
            for (size_t i = 0; i < total; ++i) img.pixels[i] = to8(canvas[i], bd);
        }
    } else if (ct == 2) {
        if (has_trns) {
            img.format = kFmtRGBA8;
            img.pixels.assign(total * 4, 0);
            for (size_t i = 0; i < total; ++i) {
                const uint16_t r = canvas[3 * i], g = canvas[3 * i + 1], b = canvas[3 * i + 2];
                out4(i, to8(r, bd), to8(g, bd), to8(b, bd), (r == tr && g == tgr && b == tb) ? 0 : 255);
            }
        } else {
            img.format = kFmtRGB8;
            img.pixels.assign(total * 3, 0);
            for (size_t i = 0; i < total * 3; ++i) img.pixels[i] = to8(canvas[i], bd);
        }
    } else if (ct == 3) {
        const size_t npal = plte.size() / 3;
        img.format = has_trns ? kFmtRGBA8 : kFmtRGB8;
        img.pixels.assign(total * (has_trns ? 4 : 3), 0);
        for (size_t i = 0; i < total; ++i) {
            const uint16_t k = canvas[i];
            if (k >= npal) { err = "png: palette index out of range"; return false; }
            if (has_trns) out4(i, plte[3 * k], plte[3 * k + 1], plte[3 * k + 2], k < trns.size() ? trns[k] : 255);
            else for (int c = 0; c < 3; ++c) img.pixels[3 * i + c] = plte[3 * k + c];
        }
    } else if (ct == 4) {
        img.format = kFmtRGBA8;
        img.pixels.assign(total * 4, 0);
        for (size_t i = 0; i < total; ++i) {
            const uint8_t v = to8(canvas[2 * i], bd);
            out4(i, v, v, v, to8(canvas[2 * i + 1], bd));
        }
    } else {
        img.format = kFmtRGBA8;
        img.pixels.assign(total * 4, 0);
        for (size_t i = 0; i < total * 4; ++i) img.pixels[i] = to8(canvas[i], bd);
    }
    return true;
}

}  // namespace pb
