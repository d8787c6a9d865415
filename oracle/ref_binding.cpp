// ref_binding.cpp -- Python binding of the reference's own CUDA launchers, for
// checking against on a GPU.  TEST INFRASTRUCTURE ONLY.
//
// The reference (KudaHitamCUDA.cu) defines ultra_fused_full_fusion_cuda
// (:197-231) but never exports it (its module, :799-804, binds only forward,
// the HBBA encoder and calibrator, and fused_asymmetric_attention).  This
// file declares the launchers this engine is checked against -- with the
// reference's signatures -- and exports them from a module of its own, so the
// reference kernels can run unchanged beside the engine.  (The HBBA encoder
// is not exported: it reduces its sums within one warp of its 256 threads
// and copies its packed bytes out without a barrier, KudaHitamCUDA.cu:312-381,
// so its output is not a checker.)  build_ref.py
// compiles KudaHitamCUDA.cu where it lies and links it with this file into
// oracle/_ref/kh_ref.so.
#include <torch/extension.h>

#include <vector>

std::vector<torch::Tensor> ultra_fused_full_fusion_cuda(torch::Tensor x, torch::Tensor d,
                                                        torch::Tensor centroids);
void fwht_cuda_forward(torch::Tensor x);
torch::Tensor hbba_calibrate_cuda(torch::Tensor sample, torch::Tensor n_map, int layer_id,
                                  uint8_t active_mask);
torch::Tensor fused_asymmetric_attention_packed_cuda(torch::Tensor q, torch::Tensor k_packed,
                                                     torch::Tensor signs, torch::Tensor d_vec,
                                                     torch::Tensor k_norms, torch::Tensor r_norms,
                                                     torch::Tensor centroids, int layer_id,
                                                     uint8_t active_mask, float scale);

PYBIND11_MODULE(kh_ref, m) {
  m.def("ultra_fused_full_fusion", &ultra_fused_full_fusion_cuda,
        "reference kernel v8 (KudaHitamCUDA.cu:13-231)");
  m.def("forward", &fwht_cuda_forward, "reference orthonormal FWHT (KudaHitamCUDA.cu:233-283)");
  m.def("fused_asymmetric_attention", &fused_asymmetric_attention_packed_cuda,
        "reference packed scorer (KudaHitamCUDA.cu:695-797)");
  m.def("hbba_calibrate_cuda", &hbba_calibrate_cuda,
        "reference HBBA calibrator (KudaHitamCUDA.cu:423-516)");
}
