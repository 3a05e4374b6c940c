/* Line-image preprocessing on the device: the pixel part of the reference's
 * load_image_q (src/main.rs:218-239), for a whole batch at once.
 *
 * The reference decodes each file with the `image` crate, converts it to
 * RGB8, resizes it keeping the aspect ratio with
 * image::imageops::resize(.., FilterType::Triangle) (image 0.24.9), pastes
 * it on a white img_h x img_w canvas (left-aligned, vertically centred) and
 * maps every byte p to round(((p / 255) * 2 - 1) * 127) clamped to +-127.
 * Decoding stays on the host (it is file-format work); everything after it
 * runs here, one CTA per canvas row.  The output keeps the reference's byte
 * order, [image][y][x][rgb], which the model reads as its [3, H, W] input
 * exactly as the reference's does.
 *
 * Errors follow the library policy (trba_last_error / abort on error);
 * functions return 0 on success, -1 on a bad argument. */
#ifndef TRBA_PREPROC_H
#define TRBA_PREPROC_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* rgb: device bytes of n decoded RGB8 images, image i at byte offset
 * offsets[i] (device array), widths[i] x heights[i] pixels, rows of
 * widths[i] * 3 bytes; out: device int8 [n, img_h * img_w * 3].
 * Replaces the per-image load_image_q (src/main.rs:220-239) after
 * image::open(..).to_rgb8(). */
int trba_preprocess_lines(const uint8_t *rgb, const long long *offsets, const int *widths, const int *heights, int n,
                          int img_h, int img_w, int8_t *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif
