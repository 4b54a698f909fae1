"""Alelyon Compute Kit, vq4/v1 on B200 (sm_100a).

A drop-in for the reference package's vq4 path: `ack` (the C-ABI binding:
`Device`, `Buffer`, errors), `vq` (`VQArray`, `encode`, `fit_codebook`,
`VQDevice`, `VQAdamW`), `expert_bank` and `harness`; plus `cuda` (the same
operations on device-resident PyTorch tensors) and `parallel` (sharding
across GPUs). Importing the package loads no library and opens no device.
"""
__version__ = "0.1.0"

__all__ = ["__version__"]
