"""Readers for the reference's fixture formats (tools/test_quants.c:1-13)."""
import struct
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
SQFX, SQLX = 0x58465153, 0x584C5153


def read_fixture(path):
    b = Path(path).read_bytes()
    magic = struct.unpack_from("<I", b, 0)[0]
    if magic == SQFX:
        _, ver, t, nb, be, bb = struct.unpack_from("<6I", b, 0)
        o = 24
        raw = np.frombuffer(b, np.uint8, nb * bb, o).copy()
        o += nb * bb
        exp = np.frombuffer(b, np.float32, nb * be, o).copy()
        return {"kind": "sqfx", "type": t, "n_blocks": nb, "block_elems": be, "block_bytes": bb, "raw": raw,
                "expect": exp}
    if magic == SQLX:
        _, ver, t, out_dim, in_dim = struct.unpack_from("<5I", b, 0)
        return {"kind": "sqlx", "type": t, "out": out_dim, "in": in_dim, "blob": b[20:]}
    raise ValueError(f"{path}: unknown magic {magic:#x}")


def sqlx_parts(fx, row_bytes):
    b = fx["blob"]
    nw = row_bytes * fx["out"]
    w = np.frombuffer(b, np.uint8, nw, 0).copy()
    x = np.frombuffer(b, np.float32, fx["in"], nw).copy()
    y = np.frombuffer(b, np.float32, fx["out"], nw + 4 * fx["in"]).copy()
    return w, x, y


def golden_files(kind):
    return sorted(GOLDEN.glob(f"{kind}_*.bin"))
