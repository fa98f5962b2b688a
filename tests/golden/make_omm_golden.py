"""Writes the .omm fixtures: model files saved by the reference's own ModelSerializer.

Builds a tiny model from the reference's modules (Conv2d 3->4 3x3 with bias, BatchNorm2d(4),
Linear(4, 3); oracle/ref_shim.cpp TinyNet) in the reference engine (oracle/_ref/libomref.so,
`make -C oracle ref`), sets every parameter and buffer to seeded values, and saves it with
ModelSerializer::save (format v5) twice: plain (tiny_ref.omm) and encrypted with the password
"omb-fixture" (tiny_ref_enc.omm). tiny_ref_omm.npz holds the values that were saved, by name.

    python tests/golden/make_omm_golden.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as orc  # noqa: E402

PASSWORD = "omb-fixture"


def main():
    L = orc.ref()
    if L is None:
        raise SystemExit("oracle/_ref/libomref.so is not built (make -C oracle ref)")
    h = L.omref_model_create(3, 3)
    rng = np.random.default_rng(2026)
    saved = {}
    for kind, count, info, setter in (
            ("param", L.omref_model_num_params(h), L.omref_model_param_info, L.omref_model_set_param),
            ("buffer", L.omref_model_num_buffers(h), L.omref_model_buffer_info,
             L.omref_model_set_buffer)):
        for i in range(count):
            name = ctypes.create_string_buffer(256)
            shape = (ctypes.c_int * 4)()
            rank = info(h, i, name, 256, shape)
            dims = tuple(shape[j] for j in range(rank))
            a = rng.standard_normal(dims).astype(np.float32)
            if name.value.decode().endswith("running_var"):
                a = np.abs(a) + 0.5
            setter(h, i, a.ctypes.data)
            saved[f"{kind}:{name.value.decode()}"] = a
    for fname, pw in (("tiny_ref.omm", b""), ("tiny_ref_enc.omm", PASSWORD.encode())):
        if L.omref_model_save(h, os.path.join(HERE, fname).encode(), pw) != 0:
            raise SystemExit("ModelSerializer::save failed")
    L.omref_model_destroy(h)
    np.savez(os.path.join(HERE, "tiny_ref_omm.npz"), **saved)
    print("wrote", sorted(saved))


if __name__ == "__main__":
    main()
