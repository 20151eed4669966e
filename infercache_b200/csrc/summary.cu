// Kernel C: summary-pass scorer.  Entry point validated here; the tcgen05
// kernel is not built yet, so the call reports IC_ERR_UNSUPPORTED.
#include "common.cuh"

extern "C" int ic_summary_score(const ic_summary_args* a, void* stream) {
  (void)stream;
  if (!a) return IC_ERR_INVALID_ARG;
  ic::set_last_error("summary_score: not built in this version");
  return IC_ERR_UNSUPPORTED;
}
