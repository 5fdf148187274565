"""asu_mapped_copy: host <-> device (and device <-> device) copies done by the SMs through the host
mapping, byte for byte equal to torch's copy at every unit width (16-, 4- and 1-byte paths chosen
by the alignment of both pointers and the size), with the argument checks."""

import pytest
import torch

from asu_ascend_b200.host_pool import mapped_copy_

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _load():
    import asu_ascend_b200

    asu_ascend_b200.load()


@pytest.mark.parametrize("nbytes", [1, 3, 4, 15, 16, 48, 4096, (1 << 20) + 12, 3 << 20])
@pytest.mark.parametrize("offset", [0, 1, 4, 16])
def test_mapped_copy_matches_torch_both_directions(nbytes, offset):
    _load()
    g = torch.Generator().manual_seed(nbytes * 7 + offset)
    host_src = torch.empty(nbytes + 64, dtype=torch.uint8).pin_memory()
    host_src.copy_(torch.randint(0, 256, (nbytes + 64,), dtype=torch.uint8, generator=g))
    host_dst = torch.zeros(nbytes + 64, dtype=torch.uint8).pin_memory()
    dev_buf = torch.zeros(nbytes + 64, dtype=torch.uint8, device=DEV)
    # upload: host[offset:] -> device[offset:]
    mapped_copy_(dev_buf[offset:offset + nbytes], host_src[offset:offset + nbytes])
    torch.cuda.synchronize()
    assert torch.equal(dev_buf[offset:offset + nbytes].cpu(), host_src[offset:offset + nbytes])
    assert int(dev_buf[:offset].sum()) == 0 and int(dev_buf[offset + nbytes:].sum()) == 0  # nothing outside
    # read-back: device -> host at another offset
    o2 = (offset + 4) % 32
    mapped_copy_(host_dst[o2:o2 + nbytes], dev_buf[offset:offset + nbytes])
    torch.cuda.synchronize()
    assert torch.equal(host_dst[o2:o2 + nbytes], host_src[offset:offset + nbytes])
    assert int(host_dst[:o2].sum()) == 0 and int(host_dst[o2 + nbytes:].sum()) == 0
    # device -> device
    other = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    mapped_copy_(other, dev_buf[offset:offset + nbytes])
    torch.cuda.synchronize()
    assert torch.equal(other.cpu(), host_src[offset:offset + nbytes])


def test_mapped_copy_typed_tensors_and_streams():
    _load()
    q = torch.randint(0, 1 << 30, (128, 2048), dtype=torch.int32).pin_memory()
    d = torch.empty((128, 2048), dtype=torch.int32, device=DEV)
    s = torch.cuda.Stream(device=DEV)
    with torch.cuda.stream(s):
        mapped_copy_(d, q)
    s.synchronize()
    assert torch.equal(d.cpu(), q)
    hit = (d % 3 == 0)
    back = torch.empty((128, 2048), dtype=torch.bool).pin_memory()
    mapped_copy_(back, hit, stream=s)
    s.synchronize()
    assert torch.equal(back, hit.cpu())


def test_mapped_copy_rejects_bad_arguments():
    _load()
    from asu_ascend_b200._lib import AsuError

    d = torch.zeros(64, dtype=torch.uint8, device=DEV)
    with pytest.raises(AsuError):
        mapped_copy_(d[8:40], d[0:32])  # overlapping ranges
    with pytest.raises(RuntimeError):
        mapped_copy_(d[:16], torch.zeros(16, dtype=torch.uint8))  # host memory that is not pinned
    with pytest.raises(RuntimeError):
        mapped_copy_(d[:16], d[16:48])  # sizes differ
    with pytest.raises(RuntimeError):
        mapped_copy_(torch.zeros(4).pin_memory(), torch.zeros(4).pin_memory())  # no CUDA side
