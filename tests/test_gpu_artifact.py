"""A model loaded from vae.safetensors decodes exactly as one built from the
same in-memory tensors."""
import numpy as np
import pytest
import torch

from osor_b200 import workloads
from osor_b200.artifact import write_safetensors
from osor_b200.model import NativeModel
from osor_b200.weights import random_vae_weights

pytestmark = pytest.mark.gpu


def test_model_from_safetensors_matches_in_memory(cuda_device, tmp_path):
    w = random_vae_weights(0, parts=("decoder",))
    path = str(tmp_path / "vae.safetensors")
    write_safetensors(path, w, "F32")
    lat = torch.from_numpy(workloads.decoder_latents(1, 16, 16, seed=3)).cuda()
    a = NativeModel(w, device=0, parts=("decoder",)).decode(lat)
    b = NativeModel.from_safetensors(path, device=0, parts=("decoder",)).decode(lat)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
