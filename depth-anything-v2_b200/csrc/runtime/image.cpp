#include "image.h"

#include <algorithm>
#include <cmath>
#include <stdexcept>

namespace dav2 {

ImageShape network_shape(int width, int height, int input_size) {
    if (width <= 0 || height <= 0 || input_size <= 0)
        throw std::invalid_argument("image dimensions and input_size must be positive");
    const double scale = std::max(double(input_size) / height, double(input_size) / width);
    // numpy.round (ties to even) == nearbyint in the default rounding mode
    int h = static_cast<int>(std::nearbyint(scale * height / 14.0)) * 14;
    int w = static_cast<int>(std::nearbyint(scale * width / 14.0)) * 14;
    h = std::max(h, input_size);
    w = std::max(w, input_size);
    if (h % 14) h = (h + 13) / 14 * 14;
    if (w % 14) w = (w + 13) / 14 * 14;
    return {w, h};
}

void preprocess_inferbridge_bgra8(const std::uint8_t* src, int width, int height, std::ptrdiff_t stride,
                                  ImageShape dst, std::vector<float>& out) {
    if (!src || width <= 0 || height <= 0 || stride < std::ptrdiff_t(width) * 4 || dst.width <= 0 || dst.height <= 0)
        throw std::invalid_argument("invalid InferBridge source image");
    static const float mean[3] = {0.485f, 0.456f, 0.406f};
    static const float dev[3] = {0.229f, 0.224f, 0.225f};
    const std::size_t plane = std::size_t(dst.width) * dst.height;
    out.resize(plane * 3);
    const float sx = float(width) / dst.width, sy = float(height) / dst.height;
    for (int y = 0; y < dst.height; ++y) {
        const int iy = std::min(int(std::floor(y * sy)), height - 1);
        const std::uint8_t* row = src + std::ptrdiff_t(iy) * stride;
        for (int x = 0; x < dst.width; ++x) {
            const int ix = std::min(int(std::floor(x * sx)), width - 1);
            const std::uint8_t* p = row + std::ptrdiff_t(ix) * 4;
            for (int c = 0; c < 3; ++c)
                out[std::size_t(c) * plane + std::size_t(y) * dst.width + x] = (float(p[c]) / 255.0f - mean[c]) / dev[c];
        }
    }
}

}  // namespace dav2
