// compat/src/b2_compat.h -- status-to-exception bridge shared by the
// compatibility headers: a non-zero b2engine status becomes the
// std::runtime_error the reference's CUDA_CHECK throws
// (src/common/cuda_utils.h:12-21), with b2engine's detail text appended.
#pragma once

#include <stdexcept>
#include <string>

#include "../../../include/b2engine.h"

namespace engine {
namespace cuda {

inline void b2_check(int status, const char* what) {
    if (status != 0) {
        std::string msg = std::string("b2engine ") + what + ": " + b2_status_string(status);
        const char* detail = b2_last_error();
        if (detail && detail[0]) msg += std::string(": ") + detail;
        throw std::runtime_error(msg);
    }
}

}  // namespace cuda
}  // namespace engine
