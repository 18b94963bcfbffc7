/* pdefa_c_api.h - the pdefa_* half of libpdefa_native.so.
 *
 * Signatures and structs follow the reference pdefa/include/pdefa_c_api.h
 * (line numbers below) and the export list pdefa/pdefa.def:4-23.
 * pdefa_image_load decodes PNG and baseline JPEG files on the host (the same pixels
 * as the reference's decoders; failures return NULL with a message in
 * pdefa_last_error()). pdefa_preprocess_letterbox
 * and pdefa_prepare_for_engine letterbox on the GPU, bit-identical to the reference.
 * Box and point unmapping are implemented.
 */
#ifndef PDEFA_B200_PDEFA_C_API_H
#define PDEFA_B200_PDEFA_C_API_H

#include <stdint.h>
#include <stddef.h>
#include "engine_c_api.h"

#define PDEFA_API ENGINE_API
#define PDEFA_CALL

#ifdef __cplusplus
extern "C" {
#endif

/* ---- meta: pdefa_c_api.h:25-26 ---- */
PDEFA_API const char* PDEFA_CALL pdefa_version(void);
PDEFA_API const char* PDEFA_CALL pdefa_last_error(void);

/* ---- image: pdefa_c_api.h:29-46 ---- */
typedef struct PdefaImage PdefaImage;
typedef enum {
    PDEFA_PIXFMT_GRAY8  = 0,
    PDEFA_PIXFMT_RGB8   = 1,
    PDEFA_PIXFMT_RGBA8  = 2,
    PDEFA_PIXFMT_GRAY16 = 3
} PdefaPixelFormat;

PDEFA_API PdefaImage* PDEFA_CALL pdefa_image_load(const char* path);
PDEFA_API void        PDEFA_CALL pdefa_image_free(PdefaImage* img);
PDEFA_API int32_t PDEFA_CALL pdefa_image_width   (const PdefaImage* img);
PDEFA_API int32_t PDEFA_CALL pdefa_image_height  (const PdefaImage* img);
PDEFA_API int32_t PDEFA_CALL pdefa_image_channels(const PdefaImage* img);
PDEFA_API int32_t PDEFA_CALL pdefa_image_format  (const PdefaImage* img);
PDEFA_API const uint8_t* PDEFA_CALL pdefa_image_pixels(const PdefaImage* img, size_t* out_bytes);

/* ---- preprocess: pdefa_c_api.h:49-80 ---- */
typedef struct {
    int32_t target_w;
    int32_t target_h;
    float   scale;
    float   pad_value;
} PdefaPreprocessConfig;

typedef struct {
    int32_t target_w,  target_h;
    int32_t orig_w,    orig_h;
    int32_t pad_x,     pad_y;
    int32_t scaled_w,  scaled_h;
    float   ratio;
} PdefaPreprocessMeta;

PDEFA_API EngineStatus PDEFA_CALL pdefa_preprocess_letterbox(
    const PdefaImage* img, const PdefaPreprocessConfig* cfg,
    EngineTensor** out_tensor, PdefaPreprocessMeta* out_meta);
PDEFA_API EngineStatus PDEFA_CALL pdefa_prepare_for_engine(
    const char* path, int32_t target_w, int32_t target_h, float scale, float pad_value,
    EngineTensor** out_tensor, PdefaPreprocessMeta* out_meta);
PDEFA_API EngineStatus PDEFA_CALL pdefa_load_image_as_tensor(
    const char* image_path, int32_t target_w, int32_t target_h, EngineTensor** out_tensor);

/* ---- post-process: pdefa_c_api.h:83-91 ---- */
PDEFA_API EngineStatus PDEFA_CALL pdefa_map_box_to_original(
    const float* in_box, const PdefaPreprocessMeta* meta, float* out_box);
PDEFA_API EngineStatus PDEFA_CALL pdefa_map_point_to_original(
    float* x, float* y, const PdefaPreprocessMeta* meta);

#ifdef __cplusplus
}
#endif
#endif /* PDEFA_B200_PDEFA_C_API_H */
