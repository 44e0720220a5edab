// quail_b200._native: the C++ host runtime exposed to Python.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "native.h"

namespace py = pybind11;

PYBIND11_MODULE(_native, m) {
  m.doc() = "quail_b200 C++ host runtime: SQL parser, tokenizer, planner cost model, worker IPC";
  static py::exception<qbn::SqlError> sql_error(m, "SqlError", PyExc_ValueError);
  m.def(
      "parse_sql",
      [](const std::string& text) {
        try {
          return qbn::parse_sql(text);
        } catch (const qbn::SqlError& e) {
          std::string msg = std::string(e.what()) + " (at offset " + std::to_string(e.pos) + ")";
          PyErr_SetString(sql_error.ptr(), msg.c_str());
          throw py::error_already_set();
        }
      },
      "SQL text -> JSON syntax tree");
}
