// Link shim for the reference arm: the reference's dataset loader sources (src/dataset/**) are not in
// its snapshot, only the header.  Its LoaderBatchGuard (src/rfdetr/target_builder.cpp) names two
// loader methods; the benchmark feeds batches without the loader, so these are never reached.
#include "dataset_loader.h"

#include <stdexcept>

namespace mmltk {

void DatasetLoader::handoff_batch(const Batch&, void*) {
    throw std::runtime_error("the reference's dataset loader sources are not part of its snapshot");
}

void DatasetLoader::release_batch(const Batch&, void*) {
    throw std::runtime_error("the reference's dataset loader sources are not part of its snapshot");
}

}  // namespace mmltk
