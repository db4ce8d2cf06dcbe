// Runtime controller bindings.
#include "runtime.h"

namespace axr {
void bind_runtime(pybind11::module_& m) { (void)m; }
}  // namespace axr
