// Registration hooks for op groups that live outside csrc/ops.cpp (prefill,
// MoE, communication).  Each group adds its schemas, CUDA impls and pybind
// helpers through these three functions.
#pragma once
#include <torch/extension.h>
#include <torch/library.h>

namespace bwn {
void register_ext_defs(torch::Library& m);
void register_ext_impls(torch::Library& m);
void register_ext_pybind(pybind11::module& mod);
void register_comm_defs(torch::Library& m);
void register_comm_impls(torch::Library& m);
void register_comm_pybind(pybind11::module& mod);

// per (device, stream) split-K / split-KV scratch (defined in ops.cpp)
struct Scratch {
  at::Tensor ws;
  at::Tensor tickets;
};
Scratch& scratch_for(const at::Tensor& like, long floats, long tickets);

// MoE combine arguments shared by ops_ext.cpp and ops_comm.cpp (ops_ext.cpp)
struct MoeCombineExArgs;
MoeCombineExArgs combine_args(const at::Tensor& y, const at::Tensor& w, const at::Tensor& pos_of,
                              const c10::optional<at::Tensor>& pos_sh, const c10::optional<at::Tensor>& sg,
                              const c10::optional<at::Tensor>& shared_y, const c10::optional<at::Tensor>& shared_gate);

// shared validation helpers (defined in ops.cpp)
void check_cuda(const at::Tensor& t, const char* name);
void check_bf16(const at::Tensor& t, const char* name);
void check_f32(const at::Tensor& t, const char* name);
}  // namespace bwn
