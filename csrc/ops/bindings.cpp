// Module multi_gpu_flashattention_b200._C: the CUDA kernels and the native ring engine.
#include <torch/extension.h>

namespace mgfa {
std::vector<torch::Tensor> umma_probe(torch::Tensor a, torch::Tensor b, torch::Tensor v);
void flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, c10::optional<torch::Tensor> o,
               c10::optional<torch::Tensor> o_state, torch::Tensor lse, double scale, bool causal,
               c10::optional<torch::Tensor> q_tile_pos, c10::optional<torch::Tensor> kv_tile_pos,
               bool merge, bool final_out, torch::Tensor status, int64_t wait_limit_ns,
               int64_t variant);
size_t flash_fwd_smem_bytes();
void flash_fwd_persistent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                          torch::Tensor lse, double scale, bool causal,
                          c10::optional<torch::Tensor> q_tile_pos,
                          c10::optional<torch::Tensor> kv_tile_pos, torch::Tensor status,
                          int64_t wait_limit_ns, torch::Tensor sched, int64_t tune,
                          int64_t grid, std::vector<int64_t> seg_lens,
                          c10::optional<torch::Tensor> trace);
void legacy_partial(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos,
                    bool causal, torch::Tensor acc, torch::Tensor m, torch::Tensor l, bool merge);
void legacy_merge(torch::Tensor m_run, torch::Tensor l_run, torch::Tensor acc_run,
                  torch::Tensor m_new, torch::Tensor l_new, torch::Tensor acc_new);
void legacy_normalize(torch::Tensor acc, torch::Tensor l, torch::Tensor out,
                      c10::optional<torch::Tensor> lse, c10::optional<torch::Tensor> m);
void register_ring_engine(py::module& m);
void register_ring_engine_p(py::module& m);
void register_ring_exchange(py::module& m);
void register_ring_bwd_engine(py::module& m);
torch::Tensor fwd_timeout_probe(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                int64_t wait_limit_ns, c10::optional<torch::Tensor> status);
void flash_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
               torch::Tensor out, torch::Tensor lse, torch::Tensor dq, torch::Tensor dk,
               torch::Tensor dv, double scale, bool causal,
               c10::optional<torch::Tensor> q_tile_pos, c10::optional<torch::Tensor> kv_tile_pos,
               bool accumulate, c10::optional<torch::Tensor> lse2_in,
               c10::optional<torch::Tensor> delta_in, torch::Tensor status, int64_t wait_limit_ns);
std::vector<torch::Tensor> flash_bwd_preprocess(torch::Tensor dout, torch::Tensor out,
                                                torch::Tensor lse);
}  // namespace mgfa

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a attention kernels and ring transport";
  m.def("umma_probe", &mgfa::umma_probe, "tcgen05 self-test: (A B^T, A V, status)");
  m.def("flash_fwd", &mgfa::flash_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"),
        py::arg("o_state"), py::arg("lse"), py::arg("scale"), py::arg("causal"),
        py::arg("q_tile_pos"), py::arg("kv_tile_pos"), py::arg("merge"), py::arg("final_out"),
        py::arg("status"), py::arg("wait_limit_ns") = int64_t(2000000000),
        py::arg("variant") = int64_t(-1));
  m.def("flash_fwd_smem_bytes", &mgfa::flash_fwd_smem_bytes);
  m.def("flash_fwd_persistent", &mgfa::flash_fwd_persistent, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("scale"), py::arg("causal"),
        py::arg("q_tile_pos"), py::arg("kv_tile_pos"), py::arg("status"),
        py::arg("wait_limit_ns"), py::arg("sched"), py::arg("tune") = int64_t(-1),
        py::arg("grid") = int64_t(0), py::arg("seg_lens") = std::vector<int64_t>(),
        py::arg("trace") = py::none());
  m.def("debug_build", []() {
#ifdef MGFA_DEBUG
    return true;
#else
    return false;
#endif
  });
  m.def("legacy_partial", &mgfa::legacy_partial, py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("scale"), py::arg("q_pos"), py::arg("k_pos"), py::arg("causal"), py::arg("acc"),
        py::arg("m"), py::arg("l"), py::arg("merge"));
  m.def("legacy_merge", &mgfa::legacy_merge);
  m.def("legacy_normalize", &mgfa::legacy_normalize, py::arg("acc"), py::arg("l"),
        py::arg("out"), py::arg("lse") = py::none(), py::arg("m") = py::none());
  m.def("flash_bwd", &mgfa::flash_bwd, py::arg("dout"), py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("out"), py::arg("lse"), py::arg("dq"), py::arg("dk"), py::arg("dv"),
        py::arg("scale"), py::arg("causal"), py::arg("q_tile_pos"), py::arg("kv_tile_pos"),
        py::arg("accumulate"), py::arg("lse2") = py::none(), py::arg("delta") = py::none(),
        py::arg("status"), py::arg("wait_limit_ns") = int64_t(2000000000));
  m.def("flash_bwd_preprocess", &mgfa::flash_bwd_preprocess);
  m.def("fwd_timeout_probe", &mgfa::fwd_timeout_probe,
        "forward launch whose arrival flag is never set (bounded-wait failure path)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("wait_limit_ns"),
        py::arg("status") = py::none());
  mgfa::register_ring_engine(m);
  mgfa::register_ring_engine_p(m);
  mgfa::register_ring_exchange(m);
  mgfa::register_ring_bwd_engine(m);
}
