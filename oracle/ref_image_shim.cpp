// C entry points over the reference's own image preprocessing
// (src/image.h:20-46 / src/image.cpp of Depth-Anything-V2's native runtime),
// compiled from the reference sources where they lie into oracle/_ref/ by
// `make ref REF=<checkout>`. Test infrastructure only: tests/golden's
// generator calls it to pin the oracle's restatement (dav2_oracle.c) to the
// reference itself; nothing on the product path loads it.
#include <cstdint>
#include <cstring>
#include <exception>
#include <vector>

#include "image.h"

extern "C" {

int dav2r_network_shape(int width, int height, int input_size, int* out_w, int* out_h) {
    try {
        const dav2::ImageShape s = dav2::network_shape(width, height, input_size);
        *out_w = s.width;
        *out_h = s.height;
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

int dav2r_preprocess_bgr8(const std::uint8_t* bgr, int width, int height, std::ptrdiff_t stride, int dst_w,
                          int dst_h, float* out) {
    try {
        std::vector<float> chw;
        dav2::preprocess_bgr8(bgr, width, height, stride, dav2::ImageShape{dst_w, dst_h}, chw);
        std::memcpy(out, chw.data(), chw.size() * sizeof(float));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

int dav2r_preprocess_inferbridge_bgra8(const std::uint8_t* bgra, int width, int height, std::ptrdiff_t stride,
                                       int dst_w, int dst_h, float* out) {
    try {
        std::vector<float> chw;
        dav2::preprocess_inferbridge_bgra8(bgra, width, height, stride, dav2::ImageShape{dst_w, dst_h}, chw);
        std::memcpy(out, chw.data(), chw.size() * sizeof(float));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

}  // extern "C"
