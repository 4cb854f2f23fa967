"""Session KV file from and into device memory (yattn_sess_kv_save / _load)
against the reference's own sess_kv_save / sess_kv_load (cache.c:174-247,
from the oracle's reference build when present): byte-identical files, and
loads that fill exactly the file's rows of the device blob."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _ref_lib():
    return oracle.load("ref") if oracle.has_ref() else oracle.load("port")


@pytest.mark.parametrize("nb,kd,max_seq,pos", [
    (4, 1024, 300, 257),      # Llama-3 kv_dim, a few blocks
    (2, 4096, 8192, 8192),    # 64 MB spans: more than one staging chunk per span
    (3, 256, 64, 0),          # header only
    (1, 512, 33, 33),         # pos == max_seq
])
def test_sess_kv_matches_reference(dev, tmp_path, nb, kd, max_seq, pos):
    from yllm_b200 import attn

    lib = _ref_lib()
    n = (2 * nb + 1) * max_seq * kd
    g = torch.Generator(device=dev)
    g.manual_seed(nb * 1000 + pos)
    blob = torch.randint(-32768, 32768, (n,), dtype=torch.int32, device=dev, generator=g).to(torch.int16)
    host = blob.cpu().numpy().view(np.uint16)
    ours, ref = tmp_path / "ours.kv", tmp_path / "ref.kv"
    attn.sess_kv_save(blob, nb, kd, max_seq, pos, str(ours))
    assert lib.orc_sess_kv_save(host, nb, kd, max_seq, pos, str(ref).encode()) == 0
    assert ours.stat().st_size == ref.stat().st_size == 24 + 2 * nb * pos * kd * 2
    assert ours.read_bytes() == ref.read_bytes(), "file differs from the reference's sess_kv_save"

    back = torch.zeros(n, dtype=torch.int16, device=dev)
    assert attn.sess_kv_load(back, nb, kd, max_seq, str(ref)) == pos
    got = back.cpu().numpy().view(np.uint16).reshape(2 * nb + 1, max_seq, kd)
    want = np.zeros_like(got)
    src = host.reshape(2 * nb + 1, max_seq, kd)
    want[1:, :pos] = src[1:, :pos]
    assert np.array_equal(got, want), "load touched rows outside the file's or missed some"
    # the reference loader reads our file into the same rows
    hb = np.zeros(n, np.uint16)
    p = C.c_uint32(0)
    assert lib.orc_sess_kv_load(hb, nb, kd, max_seq, str(ours).encode(), C.byref(p)) == 0 and p.value == pos
    assert np.array_equal(hb.reshape(got.shape), want)


def test_sess_kv_load_refuses_other_geometry(dev, tmp_path):
    from yllm_b200 import attn
    from yllm_b200._lib import YattnError

    nb, kd, max_seq = 2, 128, 16
    blob = torch.ones((2 * nb + 1) * max_seq * kd, dtype=torch.int16, device=dev)
    path = tmp_path / "s.kv"
    attn.sess_kv_save(blob, nb, kd, max_seq, 5, str(path))
    other = torch.zeros((2 * (nb + 1) + 1) * max_seq * kd, dtype=torch.int16, device=dev)
    with pytest.raises(YattnError, match="n_blocks"):
        attn.sess_kv_load(other, nb + 1, kd, max_seq, str(path))
    assert int(other.abs().sum()) == 0
    data = path.read_bytes()
    (tmp_path / "t.kv").write_bytes(data[:-10])
    with pytest.raises(YattnError, match="truncated"):
        attn.sess_kv_load(blob, nb, kd, max_seq, str(tmp_path / "t.kv"))
