// Registration of the extension's non-Runtime parts (one pybind11 module).
#pragma once

#include <pybind11/pybind11.h>

namespace engram {

// ops.cpp: the standalone per-owner pack and the NVTX switch.
void bind_ops(pybind11::module_ &m);
// harness.cpp: CPU harnesses for the owner service and descriptor passing.
void bind_harness(pybind11::module_ &m);

} // namespace engram
