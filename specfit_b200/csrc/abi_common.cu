// Error reporting and device queries shared by every entry point.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"
#include "swiglu.h"
#include "tree_attn.h"

namespace sf {

static thread_local std::string g_last_error;

int set_error(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int num_sms() {
  static thread_local int cached_device = -1;
  static thread_local int cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    cached_device = dev;
    cached_sms = sms;
  }
  return cached_sms;
}

}  // namespace sf

extern "C" const char* sf_last_error(void) { return sf::g_last_error.c_str(); }

extern "C" int sf_abi_version(void) { return 1; }

extern "C" int sf_device_status(int* status, int reset) {
  using namespace sf;
  SF_CHECK_ARG(status, "null pointer argument");
  int a = 0, b = 0, c = 0;
  if (int rc = swiglu_status(&a, reset)) return rc;
  if (int rc = dense_status(&b, reset)) return rc;
  if (int rc = tree_attention_tc_status(&c, reset)) return rc;
  *status = a ? a : (b ? b : c);
  return SF_OK;
}
