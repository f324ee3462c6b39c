"""Demo / CLI (src/main.cpp of the reference): device bring-up, tensor
arithmetic, matmul and ReLU through TensorOpsStatic, a Dense layer, and a
short MLP training run, printing what ran where.

    python -m dlvk_b200 [--device cuda:0|cpu] [--train-steps 50]
"""
from __future__ import annotations

import argparse
import time


def main(argv=None) -> int:
    import torch

    import dlvk_b200 as dl
    from dlvk_b200 import runtime
    from dlvk_b200.models.sequential import Sequential
    from dlvk_b200.tensor import Tensor, TensorOpsStatic

    ap = argparse.ArgumentParser(prog="python -m dlvk_b200")
    ap.add_argument("--device", default=None)
    ap.add_argument("--train-steps", type=int, default=50)
    a = ap.parse_args(argv)
    print("dlvk_b200 - Blackwell (sm_100a) deep-learning framework demo")
    print("=" * 60)
    dev = runtime.get_device(a.device)
    print(f"device: {dev.device}  ({dev.get_device_name() if hasattr(dev, 'get_device_name') else ''})")
    A = Tensor.wrap(torch.arange(16, dtype=torch.float32).reshape(4, 4).to(dev.device))
    B = Tensor.wrap(torch.ones(4, 4, device=dev.device))
    C = Tensor.wrap(torch.empty(4, 4, device=dev.device))
    R = Tensor.wrap(torch.empty(4, 4, device=dev.device))
    TensorOpsStatic.matrix_multiply(A, B, C)
    TensorOpsStatic.relu(Tensor.wrap(C.data - 20.0), R)
    print("matmul row 0:", [float(v) for v in C.data[0]], " relu row 0:", [float(v) for v in R.data[0]])
    m = Sequential(dev, "fp32", seed=0)
    m.add_dense(784, 128).add_relu().add_dense(128, 10).add_softmax()
    m.build()
    print(m.summary())
    x = torch.rand(32, 784, generator=torch.Generator().manual_seed(0))
    y = torch.randint(0, 10, (32,), generator=torch.Generator().manual_seed(0), dtype=torch.int32)
    from dlvk_b200.training.step import TrainStep

    step = TrainStep(m, dl.CrossEntropyLoss(), dl.Adam(1e-3))
    first = float(step(x, y))
    t0 = time.perf_counter()
    for _ in range(a.train_steps):
        loss = step(x, y)
    last = float(loss)
    dt = (time.perf_counter() - t0) / max(a.train_steps, 1)
    print(f"MLP 784-128-10, batch 32, Adam: loss {first:.4f} -> {last:.4f}  ({dt * 1e3:.3f} ms/step host-timed)")
    step.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
