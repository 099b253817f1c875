// Registration of the fused tensor-parallel and model ops (b200ar._C).
#pragma once

#include <pybind11/pybind11.h>

void register_ops(pybind11::module& m);
