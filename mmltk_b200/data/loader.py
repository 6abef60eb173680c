"""Batch loader over a compiled dataset.

Wraps the native prefetching loader (``csrc/host/dataset.cpp``): the pixel
slots are pinned host tensors owned here, filled by C++ worker threads ahead of
use; ``__iter__`` yields ``(images, targets, indices)`` with the images copied
host -> device asynchronously on a dedicated copy stream and the consumer
stream waiting on an event (reference: `DatasetLoader` + `CudaStreamManager`,
`include/dataset_loader.h:29-78`, `include/cuda_stream_manager.h:15-44`).
A slot is handed back to the producer only after its copy has completed.
"""
from __future__ import annotations

from typing import Iterator, List, Optional, Tuple

import torch

from ..criterion.targets import Targets
from ..ops._ext import native

__all__ = ["CompiledDataset", "BatchLoader"]

# host slot formats: the compiled pixels are k/255, so uint8 is exact and the cheapest to upload
_FORMATS = {"float32": (0, torch.float32), "bfloat16": (1, torch.bfloat16), "uint8": (2, torch.uint8)}


class CompiledDataset:
    """Random access to a compiled ``.bin`` (memory-mapped)."""

    def __init__(self, path: str):
        self.path = path
        self.reader = native().DatasetReader(path)
        self.header = self.reader.header()

    def __len__(self):
        return self.header["num_images"]

    @property
    def class_names(self) -> List[str]:
        return list(self.header["class_names"])

    @property
    def num_classes(self) -> int:
        return self.header["num_classes"]

    @property
    def size(self) -> Tuple[int, int]:
        return self.header["width"], self.header["height"]

    def image(self, i: int) -> torch.Tensor:
        """float32 [3, H, W] in [0, 1]."""
        return self.reader.image(i)

    def instances(self, i: int):
        """(xyxy int16 [n,4] pixels, class uint8 [n], rle pair counts [n])."""
        return self.reader.instances(i)

    def targets(self, indices: List[int], slots: int) -> Tuple[Targets, torch.Tensor]:
        boxes, labels, counts, areas = self.reader.targets(list(indices), slots)
        return Targets(boxes, labels, counts, counts.tolist()), areas

    def masks(self, indices: List[int], slots: int) -> torch.Tensor:
        return self.reader.masks(list(indices), slots)


class BatchLoader:
    def __init__(self, path: str, batch_size: int, shuffle: bool = True, seed: int = 42, shard_rank: int = 0,
                 shard_count: int = 1, drop_last: bool = False, workers: int = 4, prefetch: int = 3,
                 pixels: str = "uint8", max_targets: int = 100, device: Optional[torch.device] = None,
                 with_masks: bool = False, cpus: Optional[List[int]] = None):
        self.dataset = CompiledDataset(path)
        w, h = self.dataset.size
        self.batch_size = batch_size
        if pixels not in _FORMATS:
            raise ValueError(f"pixels must be one of {sorted(_FORMATS)}")
        self.pixels = pixels
        self.max_targets = max_targets
        self.with_masks = with_masks
        self.device = device
        code, dtype = _FORMATS[pixels]
        pin = torch.cuda.is_available()
        self.slots = [torch.empty(batch_size, 3, h, w, dtype=dtype, pin_memory=pin) for _ in range(max(2, prefetch))]
        nbytes = self.slots[0].numel() * self.slots[0].element_size()
        self.loader = native().DatasetLoader(path, batch_size, shuffle, seed, shard_rank, shard_count, drop_last,
                                             workers, code, [s.data_ptr() for s in self.slots], nbytes,
                                             list(cpus or []))
        self.copy_stream = torch.cuda.Stream(device) if (device is not None and torch.device(device).type == "cuda") else None
        self.epoch = 0

    def __len__(self):
        return self.loader.num_batches()

    def set_epoch(self, epoch: int) -> None:
        self.epoch = epoch

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, Targets, List[int]]]:
        self.loader.begin_epoch(self.epoch)
        pending = None
        while True:
            item = self.loader.next()
            if item is None:
                break
            slot, idx = item
            n = len(idx)
            host = self.slots[slot][:n]
            targets, _areas = self.dataset.targets(idx, self.max_targets)
            if self.with_masks:
                targets.masks = self.dataset.masks(idx, self.max_targets).bool()
                targets.mask_offsets = [0] + list(torch.cumsum(targets.counts, 0)[:-1].tolist())
            if self.copy_stream is None:
                images = host.clone()
                self.loader.release(slot)
            else:
                cur = torch.cuda.current_stream(self.device)
                with torch.cuda.stream(self.copy_stream):
                    images = host.to(self.device, non_blocking=True)
                    targets = targets.to(self.device, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.copy_stream)
                cur.wait_event(ev)
                images.record_stream(cur)
                # the previous slot's copy has certainly finished once this one is queued behind it
                if pending is not None:
                    pending[1].synchronize()
                    self.loader.release(pending[0])
                pending = (slot, ev)
            yield images, targets, idx
        if pending is not None:
            pending[1].synchronize()
            self.loader.release(pending[0])
