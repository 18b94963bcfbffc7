// Host image decoding behind pdefa_image_load (imageloader/src/loader.cpp).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace pb {

// PdefaPixelFormat codes (pdefa/include/pdefa_c_api.h)
constexpr int kFmtGRAY8 = 0, kFmtRGB8 = 1, kFmtRGBA8 = 2, kFmtGRAY16 = 3;

struct DecodedImage {
    uint32_t width = 0, height = 0;
    int format = kFmtRGB8;
    std::vector<uint8_t> pixels;   // row-major, tightly packed
};

// PNG file bytes -> pixels; false with a message in err on malformed input.
bool decode_png(const uint8_t* data, size_t n, DecodedImage& img, std::string& err);

// Baseline JPEG file bytes -> RGB8 pixels; false with a message in err.
bool decode_jpeg(const uint8_t* data, size_t n, DecodedImage& img, std::string& err);

}  // namespace pb
