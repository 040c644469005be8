// Aggregates the per-translation-unit device error words (see MSGL_ERROR_ACCESSOR).
#include "api.h"

extern "C" int msgl_err_gemm(int* info);
extern "C" int msgl_err_elementwise(int* info);
extern "C" int msgl_err_attention(int* info);
extern "C" int msgl_err_sampling(int* info);
extern "C" int msgl_err_comm(int* info);
extern "C" int msgl_err_moe(int* info);
extern "C" int msgl_err_plan(int* info);

extern "C" int msgl_get_error(int* info) {
  int (*fns[])(int*) = {msgl_err_gemm, msgl_err_elementwise, msgl_err_attention, msgl_err_sampling, msgl_err_comm, msgl_err_moe, msgl_err_plan};
  int first = 0;
  for (auto f : fns) {
    int inf = 0;
    const int c = f(&inf);
    if (c != 0 && first == 0) {
      first = c;
      if (info) *info = inf;
    }
  }
  return first;
}
