#include "native_api.h"

namespace mmltk {
void register_eval_api(pybind11::module& m) { (void)m; }
}  // namespace mmltk
