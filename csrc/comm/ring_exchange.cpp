// Python registration of RingExchange (class in ring_exchange.hpp).
#include <torch/extension.h>

#include "ring_exchange.hpp"

namespace mgfa {

void register_ring_exchange(py::module& m) {
  py::class_<RingExchange, std::shared_ptr<RingExchange>>(m, "RingExchange")
      .def(py::init<int, int, int, int64_t, int>(), py::arg("rank"), py::arg("world"),
           py::arg("device"), py::arg("slot_bytes"), py::arg("n_ctas") = 296)
      .def("ipc_handle", [](const RingExchange& e) { return py::bytes(e.ipc_handle()); })
      .def("connect", &RingExchange::connect)
      .def("slot", &RingExchange::slot)
      .def("step", &RingExchange::step)
      .def("wait_received", &RingExchange::wait_received)
      .def("rotate", &RingExchange::rotate)
      .def("release", &RingExchange::release)
      .def("reset", &RingExchange::reset)
      .def("slot_bytes", &RingExchange::slot_bytes);
}

}  // namespace mgfa
