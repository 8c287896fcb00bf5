"""TEST INFRASTRUCTURE: writes .safetensors files (8-byte header length, JSON header,
raw little-endian tensor bytes) from numpy arrays, for the checkpoint-reading tests."""
import json
import os

import numpy as np

_DT = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2), "I64": (np.int64, 8)}


def write_safetensors(path, tensors, metadata=None):
    """tensors: name -> (dtype, array); dtype F32 / F16 / I64, or BF16 with the array
    holding uint16 bit patterns."""
    header, chunks, off = {}, [], 0
    for name, (dt, arr) in tensors.items():
        np_t, _ = _DT[dt]
        b = np.ascontiguousarray(arr, dtype=np_t).tobytes()
        header[name] = {"dtype": dt, "shape": list(np.shape(arr)), "data_offsets": [off, off + len(b)]}
        chunks.append(b)
        off += len(b)
    if metadata is not None:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(np.uint64(len(h)).tobytes())
        f.write(h)
        for c in chunks:
            f.write(c)


def write_checkpoint(dir_, base, tensors, shards=1):
    """<dir>/<base>.safetensors, or `shards` files plus <base>.safetensors.index.json."""
    os.makedirs(dir_, exist_ok=True)
    if shards == 1:
        write_safetensors(os.path.join(dir_, base + ".safetensors"), tensors)
        return
    names = list(tensors)
    weight_map = {}
    for s in range(shards):
        fname = f"{base}-{s + 1:05d}-of-{shards:05d}.safetensors"
        part = {n: tensors[n] for n in names[s::shards]}
        write_safetensors(os.path.join(dir_, fname), part)
        weight_map.update({n: fname for n in part})
    with open(os.path.join(dir_, base + ".safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
