// Declarations of every host entry point exported by the extension.
#pragma once
#include <torch/extension.h>

namespace hb {
int64_t read_and_clear_status(int64_t device);

void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, int64_t N, int64_t epi, bool a_mn, bool b_mn,
          const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux,
          const c10::optional<at::Tensor>& resid, int64_t block_n);
}  // namespace hb
