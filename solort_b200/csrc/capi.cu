// Library-wide C-ABI entry points: version, status strings, the device status word.
#include "host_util.h"

namespace solort {
int read_decode_status(unsigned* flags);
int read_prefill_status(unsigned* flags);
int read_exchange_status(unsigned* flags);
int read_store_status(unsigned* flags);
}  // namespace solort

extern "C" int solort_attn_abi_version(void) { return SOLORT_ATTN_ABI_VERSION; }

extern "C" const char* solort_attn_status_string(int code) {
  switch (code) {
    case SOLORT_OK:
      return "ok";
    case SOLORT_ERR_INVALID_ARGUMENT:
      return "invalid argument (null pointer, bad size, or misaligned pointer/stride)";
    case SOLORT_ERR_UNSUPPORTED:
      return "unsupported shape (head_dim must be 128; at most 32 query rows per KV head)";
    case SOLORT_ERR_WORKSPACE:
      return "workspace missing, misaligned or too small";
    case SOLORT_ERR_CUDA:
      return "CUDA runtime error or kernel launch failure";
    case SOLORT_ERR_TENSOR_MAP:
      return "the driver rejected a TMA tensor map";
    case SOLORT_ERR_NO_DEVICE:
      return "no sm_100 device is current";
    case SOLORT_ERR_SCRATCH_LIMIT:
      return "the call needs more split scratch than the library's static 4 MiB array; use "
             "solort_attn_decode with a workspace";
    case SOLORT_ERR_IPC:
      return "CUDA IPC export or import of an exchange buffer failed";
    default:
      return "unknown status";
  }
}

extern "C" int solort_attn_device_status(unsigned* flags) {
  if (!flags) return SOLORT_ERR_INVALID_ARGUMENT;
  *flags = 0;
  solort::DeviceInfo di;
  int rc = solort::current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  rc = solort::read_decode_status(flags);
  if (rc != SOLORT_OK) return rc;
  rc = solort::read_exchange_status(flags);
  if (rc != SOLORT_OK) return rc;
  rc = solort::read_store_status(flags);
  if (rc != SOLORT_OK) return rc;
  return solort::read_prefill_status(flags);
}
