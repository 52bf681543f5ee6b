// capi.cu -- status strings and build identification of the C-ABI.
#include "common.cuh"

extern "C" const char* b2_version(void) { return "b2engine 0.1 sm_100a"; }

extern "C" const char* b2_status_string(int status) {
    switch (status) {
        case B2_OK: return "ok";
        case B2_ERR_INVALID: return "invalid argument";
        case B2_ERR_UNSUPPORTED: return "unsupported shape or alignment";
        case B2_ERR_WORKSPACE: return "workspace too small";
        case B2_ERR_NCCL: return "NCCL error";
        case B2_ERR_STATE: return "invalid state";
        case B2_ERR_TIMEOUT: return "device wait timed out";
        default:
            if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
            return "unknown status";
    }
}
