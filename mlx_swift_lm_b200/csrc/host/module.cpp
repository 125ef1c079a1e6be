// pybind11 entry point of the host runtime (_b200host).
#include <pybind11/pybind11.h>

namespace py = pybind11;

void register_page_pool(py::module_& m);
void register_safetensors(py::module_& m);
void register_grammar(py::module_& m);
void register_grammar_pda(py::module_& m);

PYBIND11_MODULE(_b200host, m) {
  m.doc() = "B200 LM host runtime: page pool, block hashing, grammar engines (regex DFA, pushdown), safetensors IO";
  register_page_pool(m);
  register_safetensors(m);
  register_grammar(m);
  register_grammar_pda(m);
}
