"""osor_b200: B200-native (sm_100a) SDXL VAE hot path of doublesharp/osor-rs.

Host mirror of the reference's operator and backend seams over the C ABI of
``libosor_b200.so`` (include/osor_b200.h). The compute runs only in the CUDA
library; there is no CPU path.
"""
from ._lib import (Cancelled, CudaError, DeviceTimeout, InvalidArtifact, InvalidInput,
                   OsorError, Unavailable, LIB_PATH, lib)
from .weights import random_vae_weights

__all__ = ["Cancelled", "CudaError", "DeviceTimeout", "InvalidArtifact", "InvalidInput",
           "OsorError", "Unavailable", "LIB_PATH", "lib", "random_vae_weights"]
