#pragma once
// Link shim for the reference arm.  PyTorch wheels ship no ONNX protobuf headers, and the
// reference includes <onnx/onnx_pb.h> only to name ModelProto in the signatures of its ONNX
// file writer (used by NativeRfDetrModel::export_onnx, never by training or inference).  A
// forward declaration is all those signatures need.
#ifndef ONNX_NAMESPACE
#define ONNX_NAMESPACE onnx_torch
#endif

namespace ONNX_NAMESPACE {
class ModelProto;
}
