// Host-side image geometry and the InferBridge BGRA preprocessing.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace dav2 {

struct ImageShape {
    int width;
    int height;
};

// src/image.cpp:138-161: the network side length rule of the Python
// reference's Resize(keep_aspect_ratio, ensure_multiple_of=14, lower_bound).
ImageShape network_shape(int width, int height, int input_size);

// src/image.cpp:289-337: InferBridge BGRA contract — nearest (PyTorch legacy)
// resize, byte order kept as model channels, (v/255 - mean)/std in float.
void preprocess_inferbridge_bgra8(const std::uint8_t* bgra, int width, int height, std::ptrdiff_t stride,
                                  ImageShape destination, std::vector<float>& chw);

}  // namespace dav2
