"""The C++ API (libdlvk_b200.so, headers under csrc/include/dlvk/{core,tensor,
layers,loss,optimizers,model}) against the Python API on the same workload:
the reference README's model and one Adam step of the 784-128-10 MLP on
batch 32.  The C++ program (csrc/tests/cpp_api_mlp.cpp, built by _build.py
into dlvk_b200/_bin/) writes its loss, flat gradient buffer and `.dlvk`
checkpoint; this test runs the same step through the Python API and
requires all three to be bit-identical, on CPU and on a GPU."""
import os
import subprocess

import pytest
import torch

from dlvk_b200 import _build

EXE = _build.BIN_DIR / "cpp_api_mlp"


def _python_step(device, out_dir):
    import dlvk_b200 as dl
    from dlvk_b200.models.sequential import Sequential

    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        m = Sequential(device=device, seed=0)
        m.add_dense(784, 128)
        m.add_relu()
        m.add_dense(128, 10)
        m.add_softmax()
        g = torch.Generator().manual_seed(0)
        x = torch.rand(32, 784, generator=g)
        y = torch.randint(0, 10, (32,), generator=g)
        opt = dl.Adam(1e-3)
        loss = m.train_step(x, y, dl.CrossEntropyLoss(), opt)
        path = os.path.join(out_dir, "py.dlvk")
        m.save_weights(path, optimizer=opt)
        if torch.device(device).type == "cuda":
            torch.cuda.synchronize()
        loss_b = loss.detach().float().reshape(1).cpu().numpy().tobytes()
        grad_b = m.store.grad.detach().cpu().numpy().tobytes()
        with open(path, "rb") as f:
            return loss_b, grad_b, f.read()
    finally:
        torch.set_num_threads(threads)


def _cpp_step(mode, out_dir):
    assert EXE.exists(), f"{EXE} not built (run dlvk_b200._build.build())"
    r = subprocess.run([str(EXE), mode, str(out_dir)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "OK" in r.stdout
    rd = lambda n: open(os.path.join(out_dir, n), "rb").read()  # noqa: E731
    return rd("loss.bin"), rd("grad.bin"), rd("model.dlvk"), rd("model_roundtrip.dlvk")


def _check(mode, device, tmp_path):
    c_loss, c_grad, c_file, c_round = _cpp_step(mode, tmp_path)
    p_loss, p_grad, p_file = _python_step(device, str(tmp_path))
    assert c_loss == p_loss, (torch.frombuffer(bytearray(c_loss), dtype=torch.float32),
                              torch.frombuffer(bytearray(p_loss), dtype=torch.float32))
    assert len(c_grad) == len(p_grad)
    cg = torch.frombuffer(bytearray(c_grad), dtype=torch.float32)
    pg = torch.frombuffer(bytearray(p_grad), dtype=torch.float32)
    assert torch.equal(cg, pg), (cg - pg).abs().max()
    assert c_file == p_file, "C++ and Python checkpoints differ"
    assert c_round == c_file, "load + save did not reproduce the checkpoint"


def test_cpp_api_matches_python_on_cpu(tmp_path):
    _check("cpu", "cpu", tmp_path)


@pytest.mark.gpu
def test_cpp_api_matches_python_on_gpu(tmp_path):
    _check("cuda", "cuda:0", tmp_path)
