"""Readers for the fixtures written by tests/golden/make_golden.py."""
import hashlib
import json

import numpy as np

from conftest import GOLDEN


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def blockindex_small():
    z = np.load(GOLDEN / "blockindex_small.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    out = []
    for m in meta:
        k = m["key"]
        out.append((m, z[k + "_kv_idx"], z[k + "_kv_num"], z[k + "_kv_partial"]))
    return out


def blockindex_configs():
    return json.loads((GOLDEN / "blockindex_configs.json").read_text())


def perms():
    return json.loads((GOLDEN / "perm.json").read_text())


def counts():
    return json.loads((GOLDEN / "counts.json").read_text())


def attention_small():
    z = np.load(GOLDEN / "attention_small.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    return meta, z


def attention_c1():
    z = np.load(GOLDEN / "attention_c1.npz")
    return z["o"], json.loads(bytes(z["meta"]).decode())


def kernel_math():
    z = np.load(GOLDEN / "kernel_math.npz")
    return json.loads(bytes(z["cases"]).decode()), z
