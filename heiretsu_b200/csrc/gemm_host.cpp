// Torch-facing entry point of the tcgen05 GEMM: validates tensors, builds
// the TMA descriptors and picks the instantiation (gemm_inst_*.cu).
#include <ATen/cuda/CUDAContext.h>
#include <cmath>
#include <cstdlib>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "gemm_params.h"
#include "host_utils.h"
#include "ops.h"

namespace hb {

void gemm_launch_128_kk(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_128_kn(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_128_nn(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_256_kk(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_192_kk(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_192_kn(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_192_nn(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_256_kn(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);
void gemm_launch_256_nn(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const GemmParams&, cudaStream_t);

// Tensor map over a row-major bf16 matrix [rows, cols] (cols contiguous):
// box = 64 columns (one 128-byte swizzle row) x box_rows rows.
// HB_GEMM_TMA_EPILOGUE=0 selects the per-lane store epilogue (for comparisons).
static bool tma_epilogue_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("HB_GEMM_TMA_EPILOGUE");
    return !(v && v[0] == '0');
  }();
  return on;
}

// HB_GEMM_GELU selects how the activation epilogues evaluate GELU (GemmParams::gelu_mode);
// default 2 (tanh.approx), which measured 1.5% faster per GPT-2 small training step than
// the sigmoid form (20.82 vs 21.12 ms, three alternating pairs on one B200).
static int gelu_mode() {
  static const int m = [] {
    const char* v = std::getenv("HB_GEMM_GELU");
    return (v && v[0] >= '0' && v[0] <= '2') ? v[0] - '0' : 2;
  }();
  return m;
}

// (The map's element type is bf16 for either 16-bit format: loads copy bits.)
static CUtensorMap operand_map(const at::Tensor& t, int box_rows) {
  return make_tmap_2d_bf16(t.data_ptr(), t.size(1), t.size(0), t.stride(0) * 2, 64, box_rows);
}

void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, int64_t N, int64_t epi, bool a_mn, bool b_mn,
          const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux,
          const c10::optional<at::Tensor>& resid, int64_t block_n, const std::vector<uint64_t>& ag_src,
          const c10::optional<at::Tensor>& ag_flags, int64_t ag_rank, int64_t ag_rows,
          const std::vector<uint64_t>& rs_dst, int64_t rs_rank, int64_t rs_rows, int64_t grp_mode,
          const c10::optional<at::Tensor>& grp_off, int64_t grp_n, int64_t grp_b_off, int64_t grp_c_off,
          const c10::optional<at::Tensor>& drop_seed, int64_t drop_site, double drop_p, int64_t drop_row0,
          const std::vector<uint64_t>& cmb_dst, const c10::optional<at::Tensor>& cmb_inv,
          const c10::optional<at::Tensor>& cmb_w, int64_t cmb_k, int64_t cmb_n) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm: tensors must be on CUDA");
  const bool f16 = a.scalar_type() == at::kHalf;
  TORCH_CHECK((a.scalar_type() == at::kBFloat16 || f16) && b.scalar_type() == a.scalar_type(),
              "gemm: operands must be both bf16 or both fp16");
  const at::ScalarType t16 = a.scalar_type();
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm: 2-D tensors expected");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "gemm: inner dim must be contiguous");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "gemm: row strides must be multiples of 16 bytes");
  TORCH_CHECK(N % 8 == 0 && c.stride(0) % 8 == 0, "gemm: N and ldc must be multiples of 8");
  TORCH_CHECK(!(a_mn && !b_mn), "gemm: A MN-major with B K-major is not instantiated");
  c10::cuda::CUDAGuard guard(a.device());
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  TORCH_CHECK(grp_mode == 1 ? (b_mn ? b.size(0) % K == 0 : b.size(1) == K) : (b_mn ? b.size(0) : b.size(1)) == K,
              "gemm: K mismatch");
  TORCH_CHECK(grp_mode == 1 || (b_mn ? b.size(1) : b.size(0)) <= N, "gemm: B has more rows than N");
  TORCH_CHECK(c.size(0) >= M && c.size(1) >= N, "gemm: output too small");
  const bool out_bf16 = (epi == kEpiBf16 || epi == kEpiBf16Gelu || epi == kEpiBf16Dgelu);
  TORCH_CHECK(c.scalar_type() == (out_bf16 ? t16 : at::kFloat),
              "gemm: wrong output dtype for epilogue (16-bit outputs take the operands' format)");
  if (M == 0 || N == 0) return;
  if (K == 0) TORCH_CHECK(false, "gemm: K == 0 not supported");
  const int BN = (block_n == 256) ? 256 : (block_n == 192 ? 192 : 128);

  GemmParams p{};
  p.M = M;
  p.N = static_cast<int>(N);
  p.K = K;
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.status = device_status_ptr(a.get_device());
  p.f16 = f16 ? 1 : 0;
  p.gelu_mode = gelu_mode();
  if (bias && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->is_contiguous() && bias->numel() >= N && N % 4 == 0,
                "gemm: bias must be fp32 contiguous with >= N elements");
    p.bias = bias->data_ptr<float>();
  }
  if (epi == kEpiBf16Gelu || epi == kEpiBf16Dgelu) {
    TORCH_CHECK(aux && aux->defined() && aux->scalar_type() == t16 && aux->stride(1) == 1 &&
                    aux->stride(0) % 8 == 0,
                "gemm: 16-bit aux tensor (the operands' format) required");
    p.aux = aux->data_ptr();
    p.ldaux = aux->stride(0);
  }
  if (epi == kEpiF32Resid) {
    TORCH_CHECK(resid && resid->defined() && resid->scalar_type() == at::kFloat && resid->stride(1) == 1 &&
                    resid->stride(0) % 4 == 0,
                "gemm: fp32 resid tensor required");
    p.resid = resid->data_ptr<float>();
    p.ldr = resid->stride(0);
  }
  p.drop = DropoutArgs{nullptr, 0, 0, 1.f, 0};
  if (drop_p > 0.0) {
    TORCH_CHECK(epi == kEpiF32Resid, "gemm: dropout is fused into the residual epilogue only");
    TORCH_CHECK(drop_p < 1.0 && drop_seed && drop_seed->defined() && drop_seed->is_cuda() &&
                    drop_seed->scalar_type() == at::kInt && drop_seed->numel() >= 1,
                "gemm: dropout needs 0 < p < 1 and an int32 device seed");
    TORCH_CHECK(N % 2 == 0, "gemm: dropout pairs columns (N must be even)");
    p.drop.seed = reinterpret_cast<const uint32_t*>(drop_seed->data_ptr<int>());
    p.drop.site = static_cast<uint32_t>(drop_site);
    p.drop.thresh = static_cast<uint32_t>(std::lround(drop_p * 65536.0));
    p.drop.scale = static_cast<float>(1.0 / (1.0 - drop_p));
    p.drop.row0 = static_cast<long>(drop_row0);
    if (p.drop.thresh == 0) p.drop.seed = nullptr;
  }
  // Rasterisation: CTAs in flight share tiles of the larger operand; the
  // smaller one is re-read from L2.
  const long n_real = b_mn ? b.size(1) : b.size(0);
  p.raster_n = (M > n_real) ? 1 : 0;
  // Split-K for fp32-output GEMMs whose tile count leaves SMs idle (few
  // tiles, long K): partial sums are added with vector atomics.
  p.splits = 1;
  const int num_kb = (K + 63) / 64;
  p.kb_per_split = num_kb;
  int e_launch = static_cast<int>(epi);
  if (grp_mode != 0) {
    TORCH_CHECK(grp_off && grp_off->defined() && grp_off->scalar_type() == at::kInt && grp_off->is_cuda() &&
                    grp_off->numel() >= grp_n + 1 && grp_n >= 1,
                "gemm: grouped mode needs int32 device offsets [groups + 1]");
    TORCH_CHECK(ag_src.empty() && rs_dst.empty(), "gemm: grouped mode excludes all-gather / reduce-scatter");
    TORCH_CHECK(grp_mode == 1 || (grp_mode == 2 && a_mn && b_mn), "gemm: grouped mode 2 is the weight-gradient layout");
    p.grp_mode = static_cast<int>(grp_mode);
    p.grp_n = static_cast<int>(grp_n);
    p.grp_off = grp_off->data_ptr<int>();
    p.grp_b_off = static_cast<int>(grp_b_off);
    p.grp_c_off = static_cast<int>(grp_c_off);
  }
  // Outputs smaller than one wave are split; larger outputs only when K is
  // long (>= 64 k-blocks per split, e.g. the lm_head dgrad over the vocabulary),
  // where the splits' bulk fp32 reduce-adds (splits x M x N x 4 bytes through
  // L2) are small next to the tail wave they remove.
  const int sms_dev = num_sms(a.get_device());
  const long tiles_mn = (long)((M + 127) / 128) * ((N + BN - 1) / BN);
  const int min_kb_per_split = (tiles_mn < sms_dev) ? 4 : 64;
  if ((epi == kEpiF32 || epi == kEpiF32Acc) && num_kb >= 2 * min_kb_per_split && ag_src.empty() &&
      rs_dst.empty() && grp_mode == 0) {
    const int sms = sms_dev;
    const long tiles = tiles_mn;
    auto eff = [&](int s) {
      const long units = tiles * s;
      const long waves = (units + sms - 1) / sms;
      return (double)units / (double)(waves * sms);
    };
    int best = 1;
    double best_eff = eff(1);
    for (int sp = 2; sp <= 16 && num_kb / sp >= min_kb_per_split; ++sp) {
      const double e = eff(sp);
      if (e > best_eff + 0.08) {
        best = sp;
        best_eff = e;
      }
    }
    if (best > 1) {
      p.kb_per_split = (num_kb + best - 1) / best;
      p.splits = (num_kb + p.kb_per_split - 1) / p.kb_per_split;
      if (epi == kEpiF32) {  // partial sums are accumulated into a zeroed output
        HB_CUDA_CHECK(cudaMemset2DAsync(c.data_ptr(), c.stride(0) * sizeof(float), 0, sizeof(float) * N, M,
                                        at::cuda::getCurrentCUDAStream()));
      }
      e_launch = kEpiF32Atomic;
    }
  }
  if (!ag_src.empty()) {
    // A = token-gathered activations [world * ag_rows, K], filled in-kernel from the peers' shards.
    TORCH_CHECK(!a_mn && ag_src.size() <= 8 && ag_flags && ag_flags->defined(), "gemm: all-gather prologue args");
    TORCH_CHECK(ag_rows % 128 == 0 && (int64_t)ag_src.size() * ag_rows == M, "gemm: all-gather rows");
    TORCH_CHECK(a.stride(0) == K, "gemm: gathered A must be dense [M, K]");
    TORCH_CHECK(ag_flags->scalar_type() == at::kInt && ag_flags->numel() >= M / 128, "gemm: ag_flags");
    TORCH_CHECK(p.splits == 1, "gemm: split-K is not combined with the all-gather prologue");
    p.ag_world = static_cast<int>(ag_src.size());
    p.ag_rank = static_cast<int>(ag_rank);
    p.ag_rows = static_cast<int>(ag_rows);
    for (size_t i = 0; i < ag_src.size(); ++i) p.ag_src[i] = reinterpret_cast<const void*>(ag_src[i]);
    p.ag_dst = a.data_ptr();
    p.ag_flags = ag_flags->data_ptr<int>();
    HB_CUDA_CHECK(cudaMemsetAsync(p.ag_flags, 0, sizeof(int) * (M / 128), at::cuda::getCurrentCUDAStream()));
  }
  if (!cmb_dst.empty()) {
    TORCH_CHECK(grp_mode == 1 && epi == kEpiBf16 && cmb_dst.size() <= 8 && cmb_k >= 1 && cmb_n >= 1,
                "gemm: the combine epilogue belongs to a row-grouped GEMM with a 16-bit output");
    TORCH_CHECK(N % 32 == 0, "gemm: the combine epilogue stores whole 32-column chunks (N % 32 == 0)");
    TORCH_CHECK(cmb_inv && cmb_inv->defined() && cmb_inv->scalar_type() == at::kInt && cmb_inv->is_cuda() &&
                    cmb_inv->numel() >= M,
                "gemm: combine needs int32 slot indices for every output row");
    TORCH_CHECK(cmb_w && cmb_w->defined() && cmb_w->scalar_type() == at::kFloat && cmb_w->is_contiguous() &&
                    cmb_w->numel() >= cmb_k * cmb_n,
                "gemm: combine needs fp32 routing weights [tokens, K]");
    for (uint64_t ptr : cmb_dst) TORCH_CHECK(ptr % 16 == 0, "gemm: combine slots must be 16-byte aligned");
    p.cmb_world = static_cast<int>(cmb_dst.size());
    p.cmb_K = static_cast<int>(cmb_k);
    p.cmb_N = static_cast<int>(cmb_n);
    p.cmb_inv = cmb_inv->data_ptr<int>();
    p.cmb_w = cmb_w->data_ptr<float>();
    for (size_t i = 0; i < cmb_dst.size(); ++i) p.cmb_dst[i] = reinterpret_cast<void*>(cmb_dst[i]);
  }
  if (!rs_dst.empty()) {
    TORCH_CHECK(rs_dst.size() <= 8 && rs_rows % 128 == 0 && (int64_t)rs_dst.size() * rs_rows == M,
                "gemm: reduce-scatter epilogue args");
    TORCH_CHECK(epi == kEpiBf16 || epi == kEpiF32, "gemm: reduce-scatter epilogue needs a plain bf16/fp32 output");
    TORCH_CHECK(p.splits == 1 && !(bias && bias->defined()), "gemm: reduce-scatter takes no bias / split-K");
    p.rs_world = static_cast<int>(rs_dst.size());
    p.rs_rank = static_cast<int>(rs_rank);
    p.rs_rows = static_cast<int>(rs_rows);
    for (size_t i = 0; i < rs_dst.size(); ++i) p.rs_dst[i] = reinterpret_cast<void*>(rs_dst[i]);
  }
  const CUtensorMap ta = operand_map(a, a_mn ? 64 : 128);
  const CUtensorMap tb = operand_map(b, b_mn ? 64 : BN);
  // Epilogue output maps (bulk tensor stores / fp32 reduce-adds of 32x32
  // chunks, swizzled like the staging tile). Peer outputs (reduce-scatter)
  // and outputs smaller than one chunk keep per-lane stores.
  CUtensorMap tc{}, tx{};
  p.tma_epi = 0;
  {
    const bool c_f32 = !(epi == kEpiBf16 || epi == kEpiBf16Gelu || epi == kEpiBf16Dgelu);
    const long esz = c_f32 ? 4 : 2;
    const long c_rows = (grp_mode == 2) ? (long)grp_n * grp_c_off : M;
    bool ok = tma_epilogue_enabled() && rs_dst.empty() && M >= 32 && N >= 32 && (grp_mode != 2 || M % 128 == 0) &&
              reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0 && (c.stride(0) * esz) % 16 == 0 &&
              c.size(0) >= c_rows && c.size(1) >= N;
    if (epi == kEpiBf16Gelu)
      ok = ok && reinterpret_cast<uintptr_t>(p.aux) % 16 == 0 && (p.ldaux * 2) % 16 == 0;
    if (ok) {
      const uint64_t cdims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(c_rows)};
      const uint64_t cstr[1] = {static_cast<uint64_t>(c.stride(0) * esz)};
      const uint32_t box[2] = {32, 32};
      const CUtensorMapDataType t16map = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
      tc = make_tmap(c_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : t16map, 2, c.data_ptr(), cdims, cstr, box,
                     c_f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
      if (epi == kEpiBf16Gelu) {
        const uint64_t xdims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
        const uint64_t xstr[1] = {static_cast<uint64_t>(p.ldaux * 2)};
        tx = make_tmap(t16map, 2, p.aux, xdims, xstr, box, CU_TENSOR_MAP_SWIZZLE_64B);
      }
      p.tma_epi = 1;
    }
  }
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const int e = e_launch;
  if (BN == 256) {
    if (!a_mn && !b_mn) gemm_launch_256_kk(e, ta, tb, tc, tx, p, s);
    else if (!a_mn) gemm_launch_256_kn(e, ta, tb, tc, tx, p, s);
    else gemm_launch_256_nn(e, ta, tb, tc, tx, p, s);
  } else if (BN == 192) {
    if (!a_mn && !b_mn) gemm_launch_192_kk(e, ta, tb, tc, tx, p, s);
    else if (!a_mn) gemm_launch_192_kn(e, ta, tb, tc, tx, p, s);
    else gemm_launch_192_nn(e, ta, tb, tc, tx, p, s);
  } else {
    if (!a_mn && !b_mn) gemm_launch_128_kk(e, ta, tb, tc, tx, p, s);
    else if (!a_mn) gemm_launch_128_kn(e, ta, tb, tc, tx, p, s);
    else gemm_launch_128_nn(e, ta, tb, tc, tx, p, s);
  }
}

}  // namespace hb
