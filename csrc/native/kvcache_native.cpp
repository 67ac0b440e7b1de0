// pybind11 registration of the native block pool and radix prefix cache (kvcache_native.h).
#include "kvcache_native.h"

#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

namespace py = pybind11;
using barq_native::BlockPool;
using barq_native::RadixCache;

void register_kvcache(py::module_& m) {
  py::class_<BlockPool>(m, "BlockPool")
      .def(py::init<int, int>())
      .def_property_readonly("n_free", &BlockPool::n_free)
      .def_property_readonly("n_used", &BlockPool::n_used)
      .def_property_readonly("num_blocks", &BlockPool::num_blocks)
      .def_property_readonly("block_size", &BlockPool::block_size)
      .def("blocks_for", &BlockPool::blocks_for)
      .def("can_allocate", &BlockPool::can_allocate)
      .def("allocate", &BlockPool::allocate)
      .def("retain", &BlockPool::retain)
      .def("release", &BlockPool::release)
      .def("ref", &BlockPool::ref)
      .def("refs", &BlockPool::refs)
      .def("free_list", &BlockPool::free_list);
  py::class_<RadixCache>(m, "RadixCache")
      .def(py::init<BlockPool&>(), py::keep_alive<1, 2>())
      .def("match", &RadixCache::match)
      .def("insert", &RadixCache::insert)
      .def("evict", &RadixCache::evict)
      .def_property_readonly("n_blocks", &RadixCache::n_blocks)
      .def_property_readonly("queries", &RadixCache::queries)
      .def_property_readonly("hits", &RadixCache::hits);
}
