// lightbulb_b200._native: host C++ runtime pieces (block manager, GGUF).
#include <torch/extension.h>

void register_block_manager(pybind11::module_& m);
void register_gguf(pybind11::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "lightbulb_b200 host runtime (paged KV block manager, GGUF reader)";
  register_block_manager(m);
  register_gguf(m);
}
