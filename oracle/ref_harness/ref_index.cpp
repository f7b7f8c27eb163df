// Reference harness and CPU baseline: the reference's own host index helper
// Make2DIndices (src/include/batch/batch_manager.h:30-51), compiled from the
// reference source tree in place by oracle/Makefile, behind a C entry point.
// TEST INFRASTRUCTURE ONLY.
//
// Make2DIndices reads range entries with Tensor::item<size_t>()
// (batch_manager.h:34-35,42-44), which libtorch does not instantiate; the one
// specialisation below forwards it to item<int64_t>() so the header links.
// The helper's known defects are left as they are: it adds the row number
// instead of row * row_stride (batch_manager.h:43-44) and returns a default
// (float) tensor (batch_manager.h:38).  Callers that want the intended flat
// indices pass row * row_stride as the row entry.
#include <torch/torch.h>

template <>
unsigned long at::Tensor::item<unsigned long>() const {
  return static_cast<unsigned long>(this->item<int64_t>());
}

#include "batch/batch_manager.h"

// ranges: n x 3 int64 {row, start, end}; out: float [cap].
// Returns 0, -1 if the result does not fit, -2 if the helper threw.
extern "C" int ref_make2d_indices(int64_t table_rows, int64_t table_cols, const int64_t *ranges, int64_t n,
                                  float *out, int64_t cap, int64_t *out_len) {
  try {
    const auto table = torch::zeros({table_rows, table_cols});
    std::vector<torch::Tensor> rs;
    rs.reserve(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) {
      auto r = torch::empty(3);  // as NextBatch builds them (batch_manager.h:97)
      r[0] = ranges[3 * i + 0];
      r[1] = ranges[3 * i + 1];
      r[2] = ranges[3 * i + 2];
      rs.push_back(r);
    }
    const auto idx = yllang::Make2DIndices(table, rs).contiguous();
    *out_len = idx.size(0);
    if (idx.size(0) > cap) return -1;
    std::memcpy(out, idx.data_ptr<float>(), static_cast<size_t>(idx.size(0)) * sizeof(float));
  } catch (const std::exception &) {
    return -2;
  }
  return 0;
}
