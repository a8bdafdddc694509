// zkv_api.cu -- library-level helpers of the C ABI (status strings, version).
#include "../../include/zkv.h"

extern "C" const char* zkv_status_string(int status) {
    switch (status) {
        case ZKV_OK: return "ok";
        case ZKV_ERR_ARG: return "invalid argument or shape";
        case ZKV_ERR_ALIGN: return "pointer or stride not aligned as required";
        case ZKV_ERR_CAPACITY: return "size exceeds a compiled limit";
        case ZKV_ERR_LAUNCH: return "CUDA launch or attribute error";
        case ZKV_ERR_UNSUPPORTED: return "unsupported configuration";
        case ZKV_ERR_TIMEOUT: return "device-side bounded wait expired";
        case ZKV_ERR_RANGE: return "device-side index outside its range";
        default: return "unknown status";
    }
}

extern "C" int zkv_version(void) { return 100; }
