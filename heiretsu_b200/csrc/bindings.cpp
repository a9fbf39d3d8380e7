// Python bindings of the heiretsu_b200 native extension (module `_C`).
#include <torch/extension.h>
#include <pybind11/stl.h>

#include "ops.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "heiretsu_b200 sm_100a kernels and runtime";
  m.def("read_and_clear_status", &hb::read_and_clear_status, "Read and clear the device status word");
  m.def("gemm", &hb::gemm, "tcgen05 GEMM with fused epilogue", py::arg("a"), py::arg("b"), py::arg("c"),
        py::arg("N"), py::arg("epi"), py::arg("a_mn"), py::arg("b_mn"), py::arg("bias") = py::none(),
        py::arg("aux") = py::none(), py::arg("resid") = py::none(), py::arg("block_n") = 128,
        py::arg("ag_src") = std::vector<uint64_t>{}, py::arg("ag_flags") = py::none(), py::arg("ag_rank") = 0,
        py::arg("ag_rows") = 0, py::arg("rs_dst") = std::vector<uint64_t>{}, py::arg("rs_rank") = 0,
        py::arg("rs_rows") = 0, py::arg("grp_mode") = 0, py::arg("grp_off") = py::none(), py::arg("grp_n") = 0,
        py::arg("grp_b_off") = 0, py::arg("grp_c_off") = 0, py::arg("drop_seed") = py::none(),
        py::arg("drop_site") = 0, py::arg("drop_p") = 0.0, py::arg("drop_row0") = 0,
        py::arg("cmb_dst") = std::vector<uint64_t>{}, py::arg("cmb_inv") = py::none(), py::arg("cmb_w") = py::none(),
        py::arg("cmb_k") = 0, py::arg("cmb_n") = 0);
  m.def("layernorm_fwd", &hb::layernorm_fwd);
  m.def("layernorm_bwd_scratch_rows", &hb::layernorm_bwd_scratch_rows);
  m.def("layernorm_bwd", &hb::layernorm_bwd, py::arg("dy"), py::arg("x"), py::arg("mean"), py::arg("rstd"),
        py::arg("w"), py::arg("dres_in"), py::arg("dres"), py::arg("dres16"), py::arg("scratch"), py::arg("dgamma"),
        py::arg("dbeta"), py::arg("dy_srcs") = 1);
  m.def("resid_sum_ln", &hb::resid_sum_ln);
  m.def("colsum_bf16", &hb::colsum_bf16);
  m.def("cross_entropy_fwd", &hb::cross_entropy_fwd);
  m.def("cross_entropy_bwd", &hb::cross_entropy_bwd);
  m.def("cross_entropy_fused", &hb::cross_entropy_fused);
  m.def("cross_entropy_rescale", &hb::cross_entropy_rescale);
  m.def("embedding_fwd", &hb::embedding_fwd);
  m.def("embedding_bwd", &hb::embedding_bwd);
  m.def("sumsq_scratch_size", &hb::sumsq_scratch_size);
  m.def("sumsq", &hb::sumsq);
  m.def("clip_coef", &hb::clip_coef, py::arg("norm2"), py::arg("max_norm"), py::arg("coef"), py::arg("norm") = py::none(),
        py::arg("loss_scale") = py::none());
  m.def("loss_scale_update", &hb::loss_scale_update);
  m.def("adamw_step", &hb::adamw_step);
  m.def("f32_to_bf16", &hb::f32_to_bf16);
  m.def("attention_set_trace", &hb::attention_set_trace);
  m.def("attention_fwd", &hb::attention_fwd, py::arg("qkv"), py::arg("B"), py::arg("T"), py::arg("nh"), py::arg("out"),
        py::arg("lse"), py::arg("drop_seed") = py::none(), py::arg("drop_site") = 0, py::arg("drop_p") = 0.0,
        py::arg("h0") = 0, py::arg("nh_total") = 0, py::arg("head_dim") = 64);
  m.def("dropout_bf16", &hb::dropout_bf16);
  m.def("attention_bwd", &hb::attention_bwd, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"),
        py::arg("B"), py::arg("T"), py::arg("nh"), py::arg("dvec"), py::arg("dq_acc"), py::arg("dqkv"),
        py::arg("drop_seed") = py::none(), py::arg("drop_site") = 0, py::arg("drop_p") = 0.0, py::arg("h0") = 0,
        py::arg("nh_total") = 0, py::arg("head_dim") = 64);
  m.def("raw_malloc", &hb::raw_malloc);
  m.def("raw_free", &hb::raw_free);
  m.def("tensor_from_ptr", &hb::tensor_from_ptr);
  m.def("ipc_handle", &hb::ipc_handle_py);
  m.def("ipc_open", &hb::ipc_open_py);
  m.def("ipc_close", &hb::ipc_close);
  m.def("dp_allreduce", &hb::dp_allreduce, py::arg("data"), py::arg("signal"), py::arg("rank"), py::arg("n"),
        py::arg("scale"), py::arg("counter"), py::arg("threads") = 512, py::arg("blocks") = 0);
  m.def("group_barrier", &hb::group_barrier);
  m.def("peer_sum", &hb::peer_sum);
  m.def("moe_route", &hb::moe_route);
  m.def("moe_gather", &hb::moe_gather, py::arg("x"), py::arg("pos"), py::arg("K"), py::arg("xp"), py::arg("off"),
        py::arg("e0"), py::arg("e1"), py::arg("inv") = py::none());
  m.def("moe_slots_reduce", &hb::moe_slots_reduce);
  m.def("moe_combine", &hb::moe_combine);
  m.def("moe_combine_bwd", &hb::moe_combine_bwd);
  m.def("moe_unpermute", &hb::moe_unpermute);
  m.def("moe_local_offsets", &hb::moe_local_offsets);
  m.def("moe_router_bwd", &hb::moe_router_bwd);
}
