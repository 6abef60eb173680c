// Link shim for the reference arm: the reference's ONNX file writer (src/rfdetr/onnx_model_io.cpp)
// needs the ONNX protobuf library, which this image lacks.  The training and inference paths the
// benchmark drives never call it; a call reports that plainly instead of writing a file.
#include "rfdetr/onnx_model_io.h"

#include <stdexcept>

namespace mmltk::rfdetr {

std::runtime_error onnx_model_io_error(const char* message, const std::filesystem::path& path) {
    return std::runtime_error(std::string(message) + ": " + path.string());
}

void write_onnx_model_proto(const std::shared_ptr<ONNX_NAMESPACE::ModelProto>&, const std::filesystem::path& path) {
    throw onnx_model_io_error("ONNX protobuf I/O is not built in the reference benchmark arm", path);
}

std::string serialize_onnx_model_proto(const std::shared_ptr<ONNX_NAMESPACE::ModelProto>&) {
    throw std::runtime_error("ONNX protobuf I/O is not built in the reference benchmark arm");
}

}  // namespace mmltk::rfdetr
