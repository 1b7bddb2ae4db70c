"""Token data: multi-source memory-mapped loader (reference semantics) and synthetic batches."""
from .loader import (build_manifest, dataloader_multi_source, resolve_source_files, MultiSourceDataset,  # noqa: F401
                     Prefetcher, synthetic_batches)
