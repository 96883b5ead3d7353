// Library-level C-ABI entry points (status strings, version).
#include "b200k.h"

extern "C" const char* b200k_status_string(int code) {
  switch (code) {
    case B200K_OK: return "ok";
    case B200K_ERR_ARG: return "invalid argument (null pointer, negative size or bad enum)";
    case B200K_ERR_ALIGN: return "alignment requirement not met (16-byte pointers / row strides)";
    case B200K_ERR_SHAPE: return "unsupported or inconsistent shape";
    case B200K_ERR_UNSUPPORTED: return "unsupported dtype, layout or tile configuration";
    case B200K_ERR_LAUNCH: return "CUDA launch failed";
    case B200K_ERR_TIMEOUT: return "device-side wait timed out";
    case B200K_ERR_PROGRAM: return "malformed epilogue program";
    case B200K_ERR_DEVICE: return "no usable CUDA device";
    default: return "unknown b200k status";
  }
}

extern "C" int b200k_version(void) { return 1; }
