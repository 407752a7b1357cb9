"""Record descriptors made by the reference's NIXL-UCX store (run in the build container).

Imports pack_desc from the reference's src/rngd_pd/connector/ucxkv.py (nothing is copied into
this repository) and writes tests/golden/ucx_desc.npz: for each case the arguments (agent
name, metadata, address, n, crc) and the descriptor bytes.  tests/test_kv_ucx.py checks that
this build packs the same bytes and reads the reference's.

    python tests/golden/make_ucx_desc.py --reference <reference checkout>   (or $RNGD_REFERENCE)
"""
import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = [("airm-kv-prefill-0", b'{"agent": "prefill", "ucx": [1, 2, 3]}', 0x7F12_3456_7000, 1 << 20, 0xDEADBEEF),
         ("p", b"", 4096, 0, 0),
         ("airm-kv-é-node-7", bytes(range(256)) * 3, 2 ** 63 + 64, 67_108_864, 1)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RNGD_REFERENCE"),
                    help="the reference project checkout (default $RNGD_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("pass --reference <reference checkout> or set RNGD_REFERENCE")
    sys.path.insert(0, os.path.join(a.reference, "src"))
    from rngd_pd.connector import ucxkv
    assert os.path.abspath(ucxkv.__file__).startswith(os.path.abspath(a.reference)), ucxkv.__file__
    out = {}
    for i, (name, md, addr, n, crc) in enumerate(CASES):
        out[f"desc{i}"] = np.frombuffer(ucxkv.pack_desc(name, md, addr, n, crc), np.uint8)
        out[f"args{i}"] = np.frombuffer(json.dumps([name, md.hex(), addr, n, crc]).encode(), np.uint8)
    path = os.path.join(HERE, "ucx_desc.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(CASES)} descriptors")


if __name__ == "__main__":
    main()
