// Host-native runtime controllers (spec-depth scheduler, memory field, metrics,
// event ring, spec plan). Their Python bindings are registered by bind_runtime().
#pragma once

#include <pybind11/pybind11.h>

namespace axr {
void bind_runtime(pybind11::module_& m);
}  // namespace axr
