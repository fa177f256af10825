"""Test-side writer of the reference's index files: a restatement of
IndexSerializer.save (format version 2) and saveMmapCompatible (version 3,
sections page-aligned), Sources/MetalANNSCore/IndexSerializer.swift:11-137,
plus version 1 (no storage-type field, read by IndexSerializer.load :141-230).
Little-endian u32 header fields; vectors, adjacency (u32), edge distances
(f32); u32 IDMap byte count, JSON IDMap, u32 entry point."""
import json
import struct

import numpy as np


def write_mann(path, vectors, degree=4, metric=0, storage=0, version=3, page_size=16384,
               entry_point=0, seed=0):
    vectors = np.asarray(vectors)
    n, dim = vectors.shape
    rng = np.random.default_rng(seed)
    adjacency = rng.integers(0, n, (n, degree), dtype=np.uint32)
    dists = rng.random((n, degree), dtype=np.float32)
    if storage == 0:
        vbytes = np.ascontiguousarray(vectors, np.float32).tobytes()
    elif storage == 1:
        vbytes = np.ascontiguousarray(vectors, np.float16).tobytes()
    else:
        vbytes = np.ascontiguousarray(vectors, np.uint8).tobytes()
        dim = vectors.shape[1] * 8
    idmap = json.dumps({"externalToInternal": {f"v{i}": i for i in range(min(n, 3))},
                        "nextID": n}).encode()
    out = bytearray(b"MANN")
    out += struct.pack("<IIIII", version, n, degree, dim, metric)
    if version >= 2:
        out += struct.pack("<I", storage)

    def pad():
        if version == 3:
            out.extend(b"\0" * ((page_size - len(out) % page_size) % page_size))

    pad()
    out += vbytes
    pad()
    out += adjacency.tobytes()
    pad()
    out += dists.tobytes()
    pad()
    out += struct.pack("<I", len(idmap)) + idmap + struct.pack("<I", entry_point)
    with open(path, "wb") as f:
        f.write(out)
    return bytes(out)
