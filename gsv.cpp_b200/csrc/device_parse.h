// device_parse.h -- device string -> CUDA ordinal for the drop-in classes (gsv_ar, gsv_bert, gsv_dit), with
// the meanings of gsv_device_parse (reference src/gsv_device.h:19-37): "N" or "anything:N" selects GPU N,
// "gpu" / "cuda" / "vulkan" GPU 0. The CUDA build has no CPU path, so "" also means GPU 0 and "cpu" is an
// error (false).
#pragma once

#include <cstdlib>
#include <string>

namespace gsvcu {

inline bool parse_device(const std::string& d, int* idx) {
    *idx = 0;
    if (d == "cpu" || d == "CPU" || d == "CPUExecutionProvider") return false;
    if (d.empty()) return true;
    const size_t colon = d.rfind(':');
    if (colon != std::string::npos) {
        *idx = std::atoi(d.c_str() + colon + 1);
        return true;
    }
    if (d.find_first_not_of("0123456789") == std::string::npos) *idx = std::atoi(d.c_str());
    return true;
}

}  // namespace gsvcu
