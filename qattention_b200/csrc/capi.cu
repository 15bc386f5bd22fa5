// Host-side helpers of the C ABI: status names and version string.
#include "../../include/qattn_b200.h"

extern "C" const char* qa_status_string(int status) {
  switch (status) {
    case QA_OK: return "ok";
    case QA_ERR_INVALID: return "invalid argument";
    case QA_ERR_UNSUPPORTED: return "unsupported head_dim/dtype";
    case QA_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case QA_ERR_LAUNCH: return "CUDA launch error";
    case QA_ERR_DEVICE: return "no usable sm_100 device";
    default: return "unknown status";
  }
}

extern "C" const char* qa_version(void) { return "qattn-b200 0.1.0 sm_100a"; }
