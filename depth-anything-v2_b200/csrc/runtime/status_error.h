// Failures that carry their public status. The reference maps its own error
// classes to dav2_status in one place (src/dav2.cpp:71-90: ApiError,
// std::invalid_argument, std::bad_alloc, everything else INTERNAL_ERROR);
// here the runtime throws StatusError where the status is known at the
// throw site (model I/O, model format, no device, device-side failure,
// unsupported request), so the C ABI never inspects message text.
#pragma once

#include <stdexcept>
#include <string>

#include "depth_anything_v2.h"

namespace dav2 {

class StatusError : public std::runtime_error {
public:
    StatusError(dav2_status status, const std::string& message) : std::runtime_error(message), status_(status) {}
    dav2_status status() const noexcept { return status_; }

private:
    dav2_status status_;
};

[[noreturn]] inline void throw_model_io(const std::string& m) { throw StatusError(DAV2_STATUS_MODEL_IO, m); }
[[noreturn]] inline void throw_model_format(const std::string& m) { throw StatusError(DAV2_STATUS_MODEL_FORMAT, m); }
[[noreturn]] inline void throw_no_device(const std::string& m) {
    throw StatusError(DAV2_STATUS_VULKAN_UNAVAILABLE, m);
}
[[noreturn]] inline void throw_inference_failed(const std::string& m) {
    throw StatusError(DAV2_STATUS_INFERENCE_FAILED, m);
}
[[noreturn]] inline void throw_unsupported(const std::string& m) { throw StatusError(DAV2_STATUS_UNSUPPORTED, m); }

}  // namespace dav2
