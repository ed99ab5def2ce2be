"""A minimal safetensors writer for the checkpoint tests (test infrastructure): 8-byte little-endian header length,
the JSON header, then the tensors' bytes back to back in the order given."""
import json

import numpy as np

DTYPE = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int32): "I32",
         np.dtype(np.int64): "I64", np.dtype(np.uint32): "U32", np.dtype(np.uint8): "U8"}


def write(path, tensors, metadata=None, header_override=None):
    """tensors: {name: array} (uint16 arrays are written as BF16 bit patterns)."""
    head = {}
    if metadata is not None:
        head["__metadata__"] = metadata
    off = 0
    blobs = []
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        dt = "BF16" if a.dtype == np.uint16 else DTYPE[a.dtype]
        head[name] = dict(dtype=dt, shape=list(a.shape), data_offsets=[off, off + a.nbytes])
        off += a.nbytes
        blobs.append(a.tobytes())
    raw = json.dumps(head).encode() if header_override is None else header_override
    with open(path, "wb") as f:
        f.write(len(raw).to_bytes(8, "little"))
        f.write(raw)
        for b in blobs:
            f.write(b)
    return raw
