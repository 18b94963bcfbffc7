// pdefa_* C ABI (pdefa/include/pdefa_c_api.h:25-91, export list pdefa/pdefa.def:4-23).
//
// Images (imageloader/): PNG files are decoded on the host (image_png.cpp, the same
// pixels as the reference's decoder); JPEG files are reported as unsupported with a
// message in pdefa_last_error(). Letterboxing runs on the GPU (letterbox.cu),
// bit-identical to imageloader/src/preprocess.cpp. The letterbox coordinate
// unmapping is implemented with the reference arithmetic
// (imageloader/src/engine_api.cpp:59-90): (v - pad) / ratio in float, clamped to
// [0, orig].
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/pdefa_b200_ext.h"
#include "image_io.h"
#include "runtime.h"

using namespace pb;

namespace {
// One error slot is shared with the engine_* half, so pdefa_last_error() (the only
// one the Python layer reads, _bindings.py:480-483) also reports engine errors.
void perr(const char* m) { pb::set_error(m); }
void perr(const std::string& m) { pb::set_error(m); }

bool read_file(const char* path, std::vector<uint8_t>& buf) {
    FILE* fp = std::fopen(path, "rb");
    if (!fp) return false;
    std::fseek(fp, 0, SEEK_END);
    const long n = std::ftell(fp);
    std::fseek(fp, 0, SEEK_SET);
    bool ok = n >= 0;
    if (ok) {
        buf.resize((size_t)n);
        ok = n == 0 || std::fread(buf.data(), 1, (size_t)n, fp) == (size_t)n;
    }
    std::fclose(fp);
    return ok;
}

// channel count the reference reports (imageloader/include/imageloader/image.hpp:20-28)
int channels_of_format(int f) { return f == kFmtRGB8 ? 3 : (f == kFmtRGBA8 ? 4 : 1); }

// Letterbox an image on the GPU (bit-identical to imageloader/src/preprocess.cpp) into
// an owned [1, 3, H, W] fp32 tensor. A 16-bit gray image goes through as the
// reference reads it: one byte per sample, rows of `width` bytes.
EngineStatus letterbox_image(const PdefaImage* img, const PdefaPreprocessConfig* cfg, EngineTensor** out,
                             PdefaPreprocessMeta* meta);
}  // namespace

struct PdefaImage {
    pb::DecodedImage im;
};

namespace {
EngineStatus letterbox_image(const PdefaImage* img, const PdefaPreprocessConfig* cfg, EngineTensor** out,
                             PdefaPreprocessMeta* meta) {
    const int ch = channels_of_format(img->im.format);
    const int W = cfg->target_w, H = cfg->target_h;
    if (W <= 0 || H <= 0) { perr("preprocess: target size must be positive"); return ENGINE_ERR_INVALID_ARG; }
    std::vector<float> buf((size_t)3 * W * H);
    PdefaPreprocessMeta m{};
    const EngineStatus rc = pdefa_letterbox(img->im.pixels.data(), 1, (int32_t)img->im.height,
                                            (int32_t)img->im.width, ch, cfg, buf.data(), &m, pb::default_device());
    if (rc != ENGINE_OK) return rc;
    const int64_t shape[4] = {1, 3, H, W};
    const EngineStatus rt = engine_tensor_create_from_data(out, shape, 4, ENGINE_F32, buf.data(), buf.size() * 4);
    if (rt != ENGINE_OK) return rt;
    if (meta) *meta = m;
    return ENGINE_OK;
}
}  // namespace

extern "C" {

PDEFA_API const char* pdefa_version(void) { return engine_version(); }
PDEFA_API const char* pdefa_last_error(void) { return engine_last_error(); }

// Decodes PNG files (image_png.cpp); JPEG files are reported as unsupported.
PDEFA_API PdefaImage* pdefa_image_load(const char* path) {
    if (!path) { perr("null arg"); return nullptr; }
    try {
        pb::clear_error();
        std::vector<uint8_t> data;
        if (!read_file(path, data)) { perr(std::string("load_image: cannot read file: ") + path); return nullptr; }
        auto img = std::make_unique<PdefaImage>();
        std::string err;
        // Format by signature, PNG first (imageloader/src/loader.cpp:12-19,60-67).
        static const uint8_t kPng[8] = {0x89, 'P', 'N', 'G', 0x0D, 0x0A, 0x1A, 0x0A};
        const uint8_t* d = data.data();
        const size_t n = data.size();
        bool ok;
        if (n < 4) { perr("load_image: file too small"); return nullptr; }
        if (n >= 8 && std::memcmp(d, kPng, 8) == 0) ok = pb::decode_png(d, n, img->im, err);
        else if (d[0] == 0xFF && d[1] == 0xD8 && d[2] == 0xFF) ok = pb::decode_jpeg(d, n, img->im, err);
        else { perr(std::string("load_image: unsupported format: ") + path); return nullptr; }
        if (!ok) { perr("load_image: " + err); return nullptr; }
        return img.release();
    } catch (const std::exception& e) {
        perr(e.what());
        return nullptr;
    }
}
PDEFA_API void pdefa_image_free(PdefaImage* img) { delete img; }
PDEFA_API int32_t pdefa_image_width(const PdefaImage* img) { return img ? (int32_t)img->im.width : 0; }
PDEFA_API int32_t pdefa_image_height(const PdefaImage* img) { return img ? (int32_t)img->im.height : 0; }
PDEFA_API int32_t pdefa_image_channels(const PdefaImage* img) { return img ? channels_of_format(img->im.format) : 0; }
PDEFA_API int32_t pdefa_image_format(const PdefaImage* img) { return img ? img->im.format : -1; }
PDEFA_API const uint8_t* pdefa_image_pixels(const PdefaImage* img, size_t* out_bytes) {
    if (!img) {
        if (out_bytes) *out_bytes = 0;
        return nullptr;
    }
    if (out_bytes) *out_bytes = img->im.pixels.size();
    return img->im.pixels.data();
}

PDEFA_API EngineStatus pdefa_preprocess_letterbox(const PdefaImage* img, const PdefaPreprocessConfig* cfg,
                                                  EngineTensor** out_tensor, PdefaPreprocessMeta* out_meta) {
    if (!img || !cfg || !out_tensor) { perr("null arg"); return ENGINE_ERR_NULL_PTR; }
    *out_tensor = nullptr;
    try {
        pb::clear_error();
        return letterbox_image(img, cfg, out_tensor, out_meta);
    } catch (const std::exception& e) {
        perr(e.what());
        return ENGINE_ERR_RUNTIME;
    }
}
PDEFA_API EngineStatus pdefa_prepare_for_engine(const char* path, int32_t target_w, int32_t target_h, float scale,
                                                float pad_value, EngineTensor** out_tensor, PdefaPreprocessMeta* out_meta) {
    if (!path || !out_tensor) { perr("null arg"); return ENGINE_ERR_NULL_PTR; }
    *out_tensor = nullptr;
    PdefaImage* img = pdefa_image_load(path);
    if (!img) return ENGINE_ERR_INVALID_ARG;
    PdefaPreprocessConfig cfg{target_w, target_h, scale, pad_value};
    const EngineStatus rc = pdefa_preprocess_letterbox(img, &cfg, out_tensor, out_meta);
    pdefa_image_free(img);
    return rc;
}
PDEFA_API EngineStatus pdefa_load_image_as_tensor(const char* image_path, int32_t target_w, int32_t target_h,
                                                  EngineTensor** out_tensor) {
    return pdefa_prepare_for_engine(image_path, target_w, target_h, 1.0f / 255.0f, 0.0f, out_tensor, nullptr);
}

PDEFA_API EngineStatus pdefa_map_box_to_original(const float* in_box, const PdefaPreprocessMeta* m, float* out_box) {
    if (!in_box || !m || !out_box) { perr("null arg"); return ENGINE_ERR_NULL_PTR; }
    auto mx = [&](float x) { float v = (x - (float)m->pad_x) / m->ratio; if (v < 0.f) v = 0.f; if (v > (float)m->orig_w) v = (float)m->orig_w; return v; };
    auto my = [&](float y) { float v = (y - (float)m->pad_y) / m->ratio; if (v < 0.f) v = 0.f; if (v > (float)m->orig_h) v = (float)m->orig_h; return v; };
    const float b0 = in_box[0], b1 = in_box[1], b2 = in_box[2], b3 = in_box[3];
    out_box[0] = mx(b0); out_box[1] = my(b1); out_box[2] = mx(b2); out_box[3] = my(b3);
    return ENGINE_OK;
}
PDEFA_API EngineStatus pdefa_map_point_to_original(float* x, float* y, const PdefaPreprocessMeta* m) {
    if (!x || !y || !m) { perr("null arg"); return ENGINE_ERR_NULL_PTR; }
    *x = (*x - (float)m->pad_x) / m->ratio;
    *y = (*y - (float)m->pad_y) / m->ratio;
    if (*x < 0.f) *x = 0.f;
    if (*y < 0.f) *y = 0.f;
    if (*x > (float)m->orig_w) *x = (float)m->orig_w;
    if (*y > (float)m->orig_h) *y = (float)m->orig_h;
    return ENGINE_OK;
}

}  // extern "C"
