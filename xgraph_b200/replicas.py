"""Index replicas across the GPUs of one node: built once, broadcast once.

Rows (request slots) are independent, so a multi-GPU deployment runs one engine per GPU,
each over its own rows, with no per-step collective.  The KG index is compiled on rank 0
and shipped to every rank once: the host-side index object (needed by `Engine` for its
checks, `anchor` and `view`) by `broadcast_object_list`, and the packed device tables by
one `broadcast` of a uint8 tensor (over NCCL and NVLink on GPUs; gloo on CPU for tests).
Each rank then creates its engine from the received device blob (`xg_create_from_device`).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Replica:
    payload: object          # what rank 0 built (for example a synthetic Workload)
    blob: object             # torch.uint8 tensor holding the packed tables, on `device`
    packed: object           # tables.PackedTables with the layout (blob array left empty on ranks > 0)


def broadcast_index(payload, packed, device, group=None) -> Replica:
    """On rank 0 pass the built payload and its PackedTables; on other ranks pass None for
    both.  Returns the same Replica on every rank: the payload object, the packed layout
    and a device tensor holding the blob, sent once from rank 0."""
    import torch
    import torch.distributed as dist

    rank = dist.get_rank(group)
    if rank == 0:
        meta = type(packed)(blob=np.zeros(0, np.uint8), layout=packed.layout, words=packed.words,
                            words_padded=packed.words_padded)
        box = [payload, meta]
    else:
        box = [None, None]
    dist.broadcast_object_list(box, src=0, group=group, device=device if device.type == "cuda" else None)
    payload, meta = box
    size = int(meta.layout.blob_bytes)
    if rank == 0:
        blob = torch.from_numpy(packed.blob).to(device)
    else:
        blob = torch.empty(size, dtype=torch.uint8, device=device)
    dist.broadcast(blob, src=0, group=group)
    return Replica(payload=payload, blob=blob, packed=packed if rank == 0 else meta)
