// gemm_3xtf32.cu — placeholder entry points for the tcgen05 contractions.
#include "kb_common.cuh"

extern "C" {

int kb_sgemm_3xtf32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t,
                    int64_t, int64_t, int, kbStream) {
  return kb::set_error(KB_ERR_UNSUPPORTED, "kb_sgemm_3xtf32: not built yet");
}
int kb_bgemm_3xtf32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t,
                    kbStream) {
  return kb::set_error(KB_ERR_UNSUPPORTED, "kb_bgemm_3xtf32: not built yet");
}
size_t kb_gemm_splitk_workspace_size(int64_t, int64_t, int64_t) { return 0; }
int kb_gemm_splitk_3xtf32(const float*, const float*, float*, int64_t, int64_t, int64_t, void*,
                          size_t, kbStream) {
  return kb::set_error(KB_ERR_UNSUPPORTED, "kb_gemm_splitk_3xtf32: not built yet");
}

}  // extern "C"
