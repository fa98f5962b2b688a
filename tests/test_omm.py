"""The .omm reader and writer (omnimatchdeeplearningtool_b200/omm.py) against files written by the
reference's own ModelSerializer::save (tests/golden/make_omm_golden.py): the values read back
are the values saved, and the writer reproduces the reference's files byte for byte, plain and
encrypted. Damaged files, missing and wrong passwords are refused. The GPU test runs an
inference plan on weights loaded from an .omm file."""
import os

import numpy as np
import pytest

from omnimatchdeeplearningtool_b200 import omm

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PASSWORD = "omb-fixture"


def _expected():
    z = np.load(os.path.join(GOLDEN, "tiny_ref_omm.npz"))
    params = {k[6:]: z[k] for k in z.files if k.startswith("param:")}
    buffers = {k[7:]: z[k] for k in z.files if k.startswith("buffer:")}
    return params, buffers


def _tiny_meta():
    return {"model_type_hash": omm.model_type_hash("TinyNet"), "num_classes": 3}


@pytest.mark.parametrize("fname,pw", [("tiny_ref.omm", None), ("tiny_ref_enc.omm", PASSWORD)])
def test_reads_reference_files(fname, pw):
    params, buffers, meta = omm.read_omm(os.path.join(GOLDEN, fname), pw)
    want_p, want_b = _expected()
    assert sorted(params) == sorted(want_p) and sorted(buffers) == sorted(want_b)
    for k, v in want_p.items():
        assert params[k].shape == v.shape and np.array_equal(params[k], v), k
    for k, v in want_b.items():
        assert np.array_equal(buffers[k], v), k
    assert meta["num_classes"] == 3 and meta["model_type_hash"] == omm.model_type_hash("TinyNet")
    assert meta["base_channels"] == 64 and meta["input_size"] == 224 and meta["in_channels"] == 3


@pytest.mark.parametrize("fname,pw", [("tiny_ref.omm", None), ("tiny_ref_enc.omm", PASSWORD)])
def test_writer_reproduces_reference_bytes(tmp_path, fname, pw):
    params, buffers, _ = omm.read_omm(os.path.join(GOLDEN, fname), pw)
    out = tmp_path / "w.omm"
    omm.write_omm(str(out), params, buffers, _tiny_meta(), version=5, password=pw)
    with open(os.path.join(GOLDEN, fname), "rb") as f:
        assert out.read_bytes() == f.read()


def test_refuses_damage_and_bad_passwords(tmp_path):
    with pytest.raises(omm.OmmError, match="password"):
        omm.read_omm(os.path.join(GOLDEN, "tiny_ref_enc.omm"))
    with pytest.raises(omm.OmmError, match="checksum"):
        omm.read_omm(os.path.join(GOLDEN, "tiny_ref_enc.omm"), "not-the-password")
    raw = bytearray(open(os.path.join(GOLDEN, "tiny_ref.omm"), "rb").read())
    raw[200] ^= 0x40
    bad = tmp_path / "bad.omm"
    bad.write_bytes(bytes(raw))
    with pytest.raises(omm.OmmError, match="checksum"):
        omm.read_omm(str(bad))
    bad.write_bytes(b"XYZ\0" + bytes(raw[4:]))
    with pytest.raises(omm.OmmError, match="magic"):
        omm.read_omm(str(bad))
    bad.write_bytes(bytes(raw[:100]))
    with pytest.raises(omm.OmmError):
        omm.read_omm(str(bad))


@pytest.mark.parametrize("version", [1, 2, 3, 4, 5])
def test_round_trip_every_version(tmp_path, version):
    params, buffers = _expected()
    bufs = buffers if version >= 2 else {}
    out = str(tmp_path / "v.omm")
    omm.write_omm(out, params, bufs, _tiny_meta(), version=version)
    p2, b2, meta = omm.read_omm(out)
    assert all(np.array_equal(p2[k], v) for k, v in params.items())
    assert all(np.array_equal(b2[k], v) for k, v in bufs.items()) and len(b2) == len(bufs)
    assert (meta is not None) == (version >= 4)


@pytest.mark.gpu
def test_plan_from_omm_weights(gpu, tmp_path):
    """A ResNet-18 plan built from weights that went through an .omm file gives the logits of
    the plan built from the same weights in memory."""
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    net = synth.resnet_spec(18)
    w = synth.make_weights(net)
    params = {k: v for k, v in w.items() if "running_" not in k}
    buffers = {k: v for k, v in w.items() if "running_" in k}
    path = str(tmp_path / "r18.omm")
    omm.write_omm(path, params, buffers, {"num_classes": 1000})
    x = synth.imagenet_input(2)
    outs = []
    for weights in (w, omm.load_weights(path)):
        plan = InferencePlan(net, weights, batch=2, dtype=_lib.DTYPE_BF16)
        outs.append(plan.run(x))
        plan.close()
    assert np.array_equal(outs[0], outs[1])
    assert gpu.kernel_error() == 0
