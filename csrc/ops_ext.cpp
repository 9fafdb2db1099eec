#include "ops_ext.h"

namespace bwn {
void register_ext_defs(torch::Library& m) {}
void register_ext_impls(torch::Library& m) {}
void register_ext_pybind(pybind11::module& mod) {}
}  // namespace bwn
