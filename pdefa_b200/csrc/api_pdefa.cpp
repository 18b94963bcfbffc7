// pdefa_* C ABI (pdefa/include/pdefa_c_api.h:25-91, export list pdefa/pdefa.def:4-23).
//
// Image decoding and letterboxing (imageloader/) are host-side IO that is not part
// of this library's GPU hot path: the image entry points report ENGINE_ERR_NOT_IMPL
// (or NULL) with an explanation in pdefa_last_error(). The letterbox coordinate
// unmapping is implemented with the reference arithmetic
// (imageloader/src/engine_api.cpp:59-90): (v - pad) / ratio in float, clamped to
// [0, orig].
#include "../../include/pdefa_c_api.h"
#include "runtime.h"

using namespace pb;

namespace {
// One error slot is shared with the engine_* half, so pdefa_last_error() (the only
// one the Python layer reads, _bindings.py:480-483) also reports engine errors.
void perr(const char* m) { pb::set_error(m); }
const char* kNoImages = "image decoding is not part of the pdefa B200 library; decode images on the host "
                        "and pass NCHW float tensors";
}  // namespace

extern "C" {

PDEFA_API const char* pdefa_version(void) { return engine_version(); }
PDEFA_API const char* pdefa_last_error(void) { return engine_last_error(); }

PDEFA_API PdefaImage* pdefa_image_load(const char* path) {
    (void)path;
    perr(kNoImages);
    return nullptr;
}
PDEFA_API void pdefa_image_free(PdefaImage* img) { (void)img; }
PDEFA_API int32_t pdefa_image_width(const PdefaImage* img) { (void)img; return 0; }
PDEFA_API int32_t pdefa_image_height(const PdefaImage* img) { (void)img; return 0; }
PDEFA_API int32_t pdefa_image_channels(const PdefaImage* img) { (void)img; return 0; }
PDEFA_API int32_t pdefa_image_format(const PdefaImage* img) { (void)img; return -1; }
PDEFA_API const uint8_t* pdefa_image_pixels(const PdefaImage* img, size_t* out_bytes) {
    (void)img;
    if (out_bytes) *out_bytes = 0;
    return nullptr;
}

PDEFA_API EngineStatus pdefa_preprocess_letterbox(const PdefaImage* img, const PdefaPreprocessConfig* cfg,
                                                  EngineTensor** out_tensor, PdefaPreprocessMeta* out_meta) {
    (void)out_meta;
    if (!img || !cfg || !out_tensor) { perr("null arg"); return ENGINE_ERR_NULL_PTR; }
    *out_tensor = nullptr;
    perr(kNoImages);
    return ENGINE_ERR_NOT_IMPL;
}
PDEFA_API EngineStatus pdefa_prepare_for_engine(const char* path, int32_t target_w, int32_t target_h, float scale,
                                                float pad_value, EngineTensor** out_tensor, PdefaPreprocessMeta* out_meta) {
    (void)target_w; (void)target_h; (void)scale; (void)pad_value; (void)out_meta;
    if (!path || !out_tensor) { perr("null arg"); return ENGINE_ERR_NULL_PTR; }
    *out_tensor = nullptr;
    perr(kNoImages);
    return ENGINE_ERR_NOT_IMPL;
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
