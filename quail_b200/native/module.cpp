// quail_b200._native: the C++ host runtime exposed to Python.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <memory>

#include "ipc.h"
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

  // ---------------------------------------------------------------- tokenizer
  py::class_<qbn::BpeTokenizer, std::shared_ptr<qbn::BpeTokenizer>>(m, "BpeTokenizer")
      .def(py::init<const std::unordered_map<std::string, int>&,
                    const std::vector<std::pair<std::string, std::string>>&,
                    const std::unordered_map<std::string, int>&, bool>(),
           py::arg("vocab"), py::arg("merges"), py::arg("added"), py::arg("ignore_merges") = false)
      .def("encode", [](qbn::BpeTokenizer& t, const std::string& text) {
        std::vector<int> ids;
        {
          py::gil_scoped_release nogil;
          ids = t.encode(text);
        }
        return ids;
      })
      .def("encode_batch", [](qbn::BpeTokenizer& t, const std::vector<std::string>& texts, int threads) {
        std::vector<std::vector<int>> out;
        {
          py::gil_scoped_release nogil;
          out = t.encode_batch(texts, threads);
        }
        return out;
      }, py::arg("texts"), py::arg("threads") = 0)
      .def("decode", [](const qbn::BpeTokenizer& t, const std::vector<int>& ids, bool skip_special) {
        return py::bytes(t.decode(ids, skip_special));
      }, py::arg("ids"), py::arg("skip_special") = false)
      .def("token_to_id", &qbn::BpeTokenizer::token_to_id)
      .def_property_readonly("vocab_size", &qbn::BpeTokenizer::vocab_size);

  // ---------------------------------------------------------------- worker IPC
  auto& ipc_error = py::register_exception<qbn::IpcError>(m, "IpcError", PyExc_OSError);
  py::register_exception<qbn::IpcTimeout>(m, "IpcTimeout", ipc_error.ptr());
  py::register_exception<qbn::IpcClosed>(m, "IpcClosed", ipc_error.ptr());
  m.def("send_frame", [](int fd, py::bytes payload, int timeout_ms) {
    std::string s = payload;
    py::gil_scoped_release nogil;
    qbn::send_frame(fd, s, timeout_ms);
  }, py::arg("fd"), py::arg("payload"), py::arg("timeout_ms") = -1);
  m.def("recv_frame", [](int fd, uint64_t max_bytes, int timeout_ms) {
    std::string s;
    {
      py::gil_scoped_release nogil;
      s = qbn::recv_frame(fd, max_bytes, timeout_ms);
    }
    return py::bytes(s);
  }, py::arg("fd"), py::arg("max_bytes") = (uint64_t)1 << 32, py::arg("timeout_ms") = -1);
  m.def("listen_unix", &qbn::listen_unix);
  m.def("accept_unix", [](int fd, int timeout_ms) {
    py::gil_scoped_release nogil;
    return qbn::accept_unix(fd, timeout_ms);
  });
  m.def("connect_unix", [](const std::string& path, int patience_ms) {
    py::gil_scoped_release nogil;
    return qbn::connect_unix(path, patience_ms);
  });
  m.def("close_fd", &qbn::close_fd);
  m.def("spawn", &qbn::spawn, py::arg("argv"), py::arg("env") = std::vector<std::string>{});
  m.def("poll_exit", &qbn::poll_exit);
  m.def("kill_pid", &qbn::kill_pid, py::arg("pid"), py::arg("sig") = 9);
  m.def("shm_write", [](const std::string& name, py::bytes b) { return qbn::shm_write(name, b); });
  m.def("unlink_path", &qbn::unlink_path);
  py::class_<qbn::MappedFile, std::shared_ptr<qbn::MappedFile>>(m, "MappedFile", py::buffer_protocol())
      .def(py::init<const std::string&>())
      .def_property_readonly("size", &qbn::MappedFile::size)
      .def_buffer([](qbn::MappedFile& f) -> py::buffer_info {
        return py::buffer_info(const_cast<void*>(f.data()), 1, py::format_descriptor<uint8_t>::format(), 1,
                               {(py::ssize_t)f.size()}, {1}, true);
      });
}
