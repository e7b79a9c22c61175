/* TEST INFRASTRUCTURE -- resolves the reference kernel file's `#include <hip/hip_runtime.h>`
 * to the host shim when that file is compiled for the CPU by oracle/ref_emulate.cpp. */
#include "../../hip_host_shim.h"
