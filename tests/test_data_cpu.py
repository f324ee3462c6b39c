"""Data subsystem on CPU: native IDX reader/writer, MNIST (files and
synthetic fallback), the native-gather DataLoader and transform oracles."""
import math

import pytest
import torch

from dlvk_b200 import _ext
from dlvk_b200.data import DataLoader, MnistDataset, SyntheticDataset, TensorDataset, TransformDataset, read_idx, \
    write_idx
from dlvk_b200.data import transforms as TF


def test_idx_roundtrip_and_endianness(tmp_path):
    t = torch.arange(-6, 6, dtype=torch.int32).reshape(3, 4) * 100000
    p = str(tmp_path / "a.idx")
    write_idx(p, t)
    raw = open(p, "rb").read()
    assert raw[:4] == bytes([0, 0, 0x0C, 2]) and raw[4:8] == (3).to_bytes(4, "big")
    assert raw[12:16] == int(t[0, 0]).to_bytes(4, "big", signed=True)
    assert torch.equal(read_idx(p), t)
    u = torch.randint(0, 256, (5, 28, 28), dtype=torch.uint8)
    write_idx(str(tmp_path / "u"), u)
    assert torch.equal(read_idx(str(tmp_path / "u")), u)


def test_mnist_files_and_fallback(tmp_path):
    imgs = torch.randint(0, 256, (7, 28, 28), dtype=torch.uint8)
    labs = torch.randint(0, 10, (7,), dtype=torch.uint8)
    write_idx(str(tmp_path / "train-images-idx3-ubyte"), imgs)
    write_idx(str(tmp_path / "train-labels-idx1-ubyte"), labs)
    ds = MnistDataset(str(tmp_path), train=True)
    assert not ds.synthetic and ds.size() == 7
    x, y = ds.get_item(3)
    assert torch.allclose(x, imgs[3].float().unsqueeze(0) / 255.0) and y == int(labs[3])
    dl = DataLoader(ds, None, batch_size=4, shuffle=False, one_hot=True)
    bx, by = dl.get_batch(1)
    assert bx.shape == (3, 1, 28, 28) and torch.allclose(bx, imgs[4:].float().unsqueeze(1) / 255.0)
    assert torch.equal(by.argmax(1), labs[4:].long()) and torch.all(by.sum(1) == 1)
    fb = MnistDataset(str(tmp_path / "none"), train=False)
    assert fb.synthetic and fb.size() == 200 and MnistDataset(str(tmp_path / "none")).size() == 1000
    assert fb.input_shape() == [1, 28, 28] and fb.num_classes() == 10


def test_permutation_deterministic_and_complete():
    D = _ext.C().data
    a, b, c = D.permutation(1000, 5, 0), D.permutation(1000, 5, 0), D.permutation(1000, 5, 1)
    assert torch.equal(a, b) and not torch.equal(a, c)
    assert torch.equal(a.sort().values, torch.arange(1000))


def test_dataloader_batches_shards_and_drop_last():
    x = torch.arange(10 * 3, dtype=torch.float32).reshape(10, 3)
    y = torch.arange(10, dtype=torch.int32) % 4
    ds = TensorDataset(x, y, 4)
    dl = DataLoader(ds, None, batch_size=4, shuffle=True, seed=3, one_hot=False, drop_last=False)
    assert dl.num_batches() == 3
    got = torch.cat([b[0] for b in dl])
    assert torch.equal(got[:, 0].sort().values, x[:, 0])
    dl2 = DataLoader(ds, None, batch_size=4, shuffle=True, seed=3, one_hot=False, drop_last=True)
    assert dl2.num_batches() == 2 and len(list(dl2)) == 2
    seen = []
    for r in range(2):
        sh = DataLoader(ds, None, batch_size=2, shuffle=True, seed=9, one_hot=False, rank=r, world_size=2)
        seen.append(torch.cat([b[1] for b in sh]).numel())
        assert sh.num_samples() == 5
    e0 = [b[0].clone() for b in dl]
    dl.new_epoch()
    e1 = [b[0].clone() for b in dl]
    assert not all(torch.equal(a, b) for a, b in zip(e0, e1))


def test_dataloader_generic_dataset_path():
    base = SyntheticDataset(9, [2, 2], 3, seed=1)
    tds = TransformDataset(base, lambda t: t * 2)
    dl = DataLoader(tds, None, batch_size=4, shuffle=False, one_hot=True)
    bx, by = dl.get_batch(0)
    assert torch.allclose(bx, base.inputs[:4] * 2) and by.shape == (4, 3)


def _img(n=3, c=2, h=5, w=6, seed=0):
    return torch.rand((n, c, h, w), generator=torch.Generator().manual_seed(seed))


def test_transform_geometry_oracles():
    x = _img()
    assert torch.equal(TF.RandomHorizontalFlip(1.0)(x), x.flip(-1))
    assert torch.equal(TF.RandomVerticalFlip(1.0)(x), x.flip(-2))
    assert torch.equal(TF.RandomHorizontalFlip(0.0)(x), x)
    assert torch.equal(TF.CenterCrop(3, 4)(x), x[:, :, 1:4, 1:5])
    rc = TF.RandomCrop(5, 6, padding=2, seed=4)(x)
    assert rc.shape == x.shape
    # every output is a shifted window of the zero-padded input
    xp = torch.nn.functional.pad(x, (2, 2, 2, 2))
    for n in range(3):
        assert any(torch.equal(rc[n], xp[n, :, i:i + 5, j:j + 6]) for i in range(5) for j in range(5))
    # rotation by 0 is the identity; by 90 degrees about (W/2, H/2) on a square image is a rotation
    sq = _img(1, 1, 4, 4)
    th0 = TF.RandomRotation.theta_for(torch.zeros(1), 4, 4)
    assert torch.equal(TF.affine_sample_reference(sq, th0, 4, 4, 1), sq)
    # resize nearest: src = floor(dst * in/out)
    rn = TF.Resize(10, 12, TF.InterpolationMode.NEAREST)(x)
    hi = (torch.arange(10) * 5 / 10).floor().long()
    wi = (torch.arange(12) * 6 / 12).floor().long()
    assert torch.equal(rn, x[:, :, hi][:, :, :, wi])
    rb = TF.Resize(5, 6)(x)
    assert torch.equal(rb, x)


def test_transform_photometric_oracles():
    x = _img()
    nm = TF.Normalize([0.5, 0.25], [0.5, 2.0])(x)
    assert torch.allclose(nm[:, 0], (x[:, 0] - 0.5) / 0.5) and torch.allclose(nm[:, 1], (x[:, 1] - 0.25) / 2.0)
    st = TF.Standardize()(x)
    flat = st.reshape(3, -1)
    assert torch.allclose(flat.mean(1), torch.zeros(3), atol=1e-6)
    assert torch.allclose(flat.pow(2).mean(1), torch.ones(3), atol=1e-5)
    mm = TF.MinMaxScale(-1.0, 2.0)(x).reshape(3, -1)
    assert torch.allclose(mm.min(1).values, torch.full((3,), -1.0)) and torch.allclose(mm.max(1).values,
                                                                                        torch.full((3,), 2.0))
    br = TF.RandomBrightness(0.3, seed=1)(x)
    assert br.min() >= 0 and br.max() <= 1
    d = (br - x).reshape(3, -1)
    inner = (x.reshape(3, -1) > 0.31) & (x.reshape(3, -1) < 0.69)
    for n in range(3):
        v = d[n][inner[n]]
        assert torch.allclose(v, v[0].expand_as(v), atol=1e-6)
    nz = TF.RandomNoise(0.1, seed=0)(torch.zeros(4, 3, 64, 64))
    assert abs(float(nz.std()) - 0.1) < 0.005
    oh = TF.ToOneHot(4)(torch.tensor([1, 3]))
    assert torch.equal(oh, torch.tensor([[0.0, 1, 0, 0], [0, 0, 0, 1]]))


def test_pipelines_and_builder():
    p = TF.create_mnist_pipeline(True)
    assert p.has_transform("normalize") and p.has_transform("random_rotation")
    y = p.process(torch.rand(2, 1, 28, 28))
    assert y.shape == (2, 1, 28, 28)
    p.remove_transform("random_rotation")
    assert not p.has_transform("random_rotation")
    b = TF.PreprocessingPipelineBuilder().resize(8, 8).random_crop(6, 6, 1).random_horizontal_flip() \
        .medium_augmentation().min_max_scale().build()
    assert b.process(torch.rand(3, 3, 10, 10)).shape == (3, 3, 6, 6)
    assert TF.create_imagenet_pipeline(False).process(torch.rand(1, 3, 230, 230)).shape == (1, 3, 224, 224)
    ra = TF.RandomApply(TF.RandomHorizontalFlip(1.0), 0.5, seed=0)
    x = _img(8)
    y = ra(x)
    flipped = [torch.equal(y[i], x[i].flip(-1)) for i in range(8)]
    kept = [torch.equal(y[i], x[i]) for i in range(8)]
    assert all(f or k for f, k in zip(flipped, kept)) and any(flipped) and any(kept)
