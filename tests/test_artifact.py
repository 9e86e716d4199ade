"""safetensors reading with the reference's file checks (src/artifact.rs:585-760),
on CPU. Files come from this package's writer and from the independent
`safetensors` package."""
import json
import struct

import numpy as np
import pytest
import torch

from osor_b200._lib import InvalidArtifact
from osor_b200.artifact import ArtifactLimits, read_safetensors, write_safetensors
from osor_b200.weights import random_vae_weights


def _small():
    rng = np.random.default_rng(0)
    return {"decoder.conv_in.weight": rng.standard_normal((8, 4, 3, 3)).astype(np.float32),
            "decoder.conv_in.bias": rng.standard_normal(8).astype(np.float32),
            "post_quant_conv.weight": rng.standard_normal((4, 4, 1, 1)).astype(np.float32)}


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
def test_round_trip(tmp_path, dtype):
    t = _small()
    p = str(tmp_path / "vae.safetensors")
    write_safetensors(p, t, dtype)
    got = read_safetensors(p)
    assert set(got) == set(t)
    for k, v in t.items():
        want = {"F32": v, "F16": v.astype(np.float16).astype(np.float32),
                "BF16": torch.from_numpy(v).to(torch.bfloat16).float().numpy()}[dtype]
        np.testing.assert_array_equal(got[k], want)
        assert got[k].dtype == np.float32 and got[k].shape == v.shape


def test_reads_files_written_by_the_safetensors_package(tmp_path):
    from safetensors.numpy import save_file
    w = random_vae_weights(0, channels=(32, 32, 64, 64), layers=1, parts=("decoder",))
    p = str(tmp_path / "vae.safetensors")
    save_file({k: v.astype(np.float16) for k, v in w.items()}, p, metadata={"format": "pt"})
    got = read_safetensors(p)
    assert set(got) == set(w)
    for k, v in w.items():
        np.testing.assert_array_equal(got[k], v.astype(np.float16).astype(np.float32))


def _raw(tmp_path, header, data=b"", header_len=None):
    head = json.dumps(header).encode()
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", len(head) if header_len is None else header_len) + head + data)
    return str(p)


@pytest.mark.parametrize("case", ["zero_header", "long_header", "gap", "overlap", "short_data",
                                  "bad_name", "empty_part", "dtype", "zero_dim", "rank",
                                  "foreign_prefix", "lora", "not_dict", "empty"])
def test_rejects_malformed_files(tmp_path, case):
    ok = {"a.weight": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}
    data = b"\0" * 8
    kw = {}
    if case == "zero_header":
        kw = dict(header_len=0)
        header = ok
    elif case == "long_header":
        kw = dict(header_len=10 ** 6)
        header = ok
    elif case == "gap":
        header = {"a.weight": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}
        data = b"\0" * 12
    elif case == "overlap":
        header = {"a.weight": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
                  "b.weight": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}
        data = b"\0" * 12
    elif case == "short_data":
        header, data = ok, b"\0" * 4
    elif case == "bad_name":
        header = {"a weight": ok["a.weight"]}
    elif case == "empty_part":
        header = {"a..weight": ok["a.weight"]}
    elif case == "dtype":
        header = {"a.weight": {"dtype": "I32", "shape": [2], "data_offsets": [0, 8]}}
    elif case == "zero_dim":
        header = {"a.weight": {"dtype": "F32", "shape": [0], "data_offsets": [0, 0]}}
        data = b""
    elif case == "rank":
        header = {"a.weight": {"dtype": "F32", "shape": [1] * 9 + [2], "data_offsets": [0, 8]}}
    elif case == "foreign_prefix":
        header = {"unet.a.weight": ok["a.weight"]}
    elif case == "lora":
        header = {"a.lora_A.weight": ok["a.weight"]}
    elif case == "not_dict":
        header = [1, 2]
    else:
        header = {}
    with pytest.raises(InvalidArtifact):
        read_safetensors(_raw(tmp_path, header, data, **kw))


def test_tensor_limit(tmp_path):
    p = str(tmp_path / "vae.safetensors")
    write_safetensors(p, _small())
    with pytest.raises(InvalidArtifact):
        read_safetensors(p, ArtifactLimits(max_tensor_bytes=100))
    with pytest.raises(InvalidArtifact):
        read_safetensors(p, ArtifactLimits(max_total_tensor_bytes=200))
