// Declarations shared by the kernel translation units and the bindings.
#pragma once

#include <torch/extension.h>
#include <cuda.h>

#include "gemm_epi.h"

namespace qb {

void gemm_sm100(const torch::Tensor& a, const torch::Tensor& b, const c10::optional<torch::Tensor>& sa,
                const c10::optional<torch::Tensor>& sb, int64_t sb_gran, int64_t epi, torch::Tensor& out,
                const c10::optional<torch::Tensor>& out_scale, const c10::optional<torch::Tensor>& residual,
                int64_t bn);

CUtensorMap make_tmap_2d(const void* ptr, CUtensorMapDataType dtype, int elem_bytes, int64_t inner,
                         int64_t outer, int64_t row_stride_elems, int box_inner, int box_outer,
                         CUtensorMapSwizzle swizzle);

int num_sms(int dev);

// A per-device int that kernels set (first writer wins) when a bounded wait
// runs out; zero means no error.
int* device_error_word(int dev);
int64_t read_and_clear_error(int64_t dev);

}  // namespace qb
