"""GPU content hash: the device tree hash equals the host one and the oracle's, for empty,
ragged and misaligned buffers and for the pixel tensor of a 4K image (42,196 patches x
1,176 fp32 values, 198 MB: what the reference hashes per warm request)."""
import numpy as np
import pytest
import torch

from oracle import content_hash as och

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [0, 1, 1000, 1024, 1025, 4097, 65537, 3 << 20, 8519757])
def test_device_hash_matches_host_and_oracle(cuda_lib, n):
    from vlcache_b200 import ops
    rng = np.random.default_rng(n)
    data = rng.integers(0, 256, n, dtype=np.uint8)
    header = np.array([1, 77, 137], np.int64).tobytes()
    ref = och.tree_hash(data, header)
    dev = torch.from_numpy(data).cuda()
    assert ops.content_hash(dev, header) == ref
    assert ops.content_hash(data, header) == ref
    if n > 8:   # a buffer that is not 16-byte aligned takes the byte-wise path
        buf = torch.zeros(n + 4, dtype=torch.uint8, device="cuda")
        buf[4:] = dev
        assert buf[4:].data_ptr() % 16 != 0
        assert ops.content_hash(buf[4:], header) == ref
    assert ops.device_error() == 0


def test_4k_image_pixels(cuda_lib):
    from vlcache_b200 import ops
    from vlcache_b200.engine.encoder_cache import compute_hash
    g = torch.Generator(device="cuda").manual_seed(4)
    px = torch.randn(42196, 1176, generator=g, device="cuda")
    grid = torch.tensor([1, 154, 274])
    key_dev = compute_hash(px, grid)
    host = px.cpu()
    assert compute_hash(host, grid) == key_dev
    assert key_dev == och.tree_hash(host.numpy().view(np.uint8), np.array([1, 154, 274], np.int64).tobytes())
    px[20000, 7] += 1.0
    assert compute_hash(px, grid) != key_dev
    assert ops.device_error() == 0
