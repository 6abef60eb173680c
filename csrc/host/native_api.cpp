#include "native_api.h"

namespace mmltk {

void register_data_api(pybind11::module& m);
void register_eval_api(pybind11::module& m);
void register_aug_api(pybind11::module& m);
void register_archive_api(pybind11::module& m);
void register_live_api(pybind11::module& m);
void register_exec_api(pybind11::module& m);

void register_native_api(pybind11::module& m) {
    register_data_api(m);
    register_eval_api(m);
    register_aug_api(m);
    register_archive_api(m);
    register_live_api(m);
    register_exec_api(m);
}

}  // namespace mmltk
