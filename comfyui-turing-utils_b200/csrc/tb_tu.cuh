// Included once by every translation unit that launches kernels: registers a
// host-side reader for this unit's device watchdog word so tb_device_error()
// can report (and clear) waits that hit their limit in any kernel.
#pragma once

#include "tb_capi_internal.h"

namespace tb {
namespace {

int tu_read_and_clear_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tb_device_error, sizeof(int)) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  if (v != 0) {
    const int zero = 0;
    (void)cudaMemcpyToSymbol(g_tb_device_error, &zero, sizeof(int));
  }
  return v;
}

struct TuErrorRegistrar {
  TuErrorRegistrar() { register_device_error_reader(&tu_read_and_clear_device_error); }
};
TuErrorRegistrar tu_error_registrar;

}  // namespace
}  // namespace tb
