"""Captures torch's CUDA LayerNorm outputs as a fixture (run on a B200).

The reference normalises with stock nn.LayerNorm on CUDA
(fast_moss/v2_runtime.py:259); this records, for a few seeded inputs, the
output, mean and rstd that torch.native_layer_norm produces on the device,
so that the CPU tests can pin oracle.layer_norm without a GPU.

Usage (on a GPU machine): python tests/golden/make_golden_gpu.py OUT.npz
"""

import sys

import numpy as np
import torch


def main(out_path):
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(20261202)
    fixture = {}
    cases = []
    for rows, n, offset in [(6, 64, 0.0), (4, 1024, 0.0), (3, 1280, 50.0), (2, 100, -7.0),
                            (2, 2048, 1e3)]:
        name = f"r{rows}_n{n}"
        x = torch.randn(rows, n, generator=g) * 2 + offset
        w = 1 + 0.1 * torch.randn(n, generator=g)
        b = 0.1 * torch.randn(n, generator=g)
        y, mean, rstd = torch.native_layer_norm(x.to(dev), (n,), w.to(dev), b.to(dev), 1e-5)
        fixture.update({
            f"{name}_x": x.numpy(), f"{name}_w": w.numpy(), f"{name}_b": b.numpy(),
            f"{name}_eps": np.float32(1e-5), f"{name}_y": y.cpu().numpy(),
            f"{name}_mean": mean.reshape(-1).cpu().numpy(),
            f"{name}_rstd": rstd.reshape(-1).cpu().numpy(),
        })
        cases.append(name)
    fixture["cases"] = np.array(cases)
    fixture["torch_version"] = np.array(torch.__version__)
    fixture["device"] = np.array(torch.cuda.get_device_name(dev))
    np.savez_compressed(out_path, **fixture)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "layer_norm_cuda.npz")
