"""opencuda-multidev (crates/opencuda-multidev/src/lib.rs) through the C ABI:
partition_layers (multidev:28-74) against a restatement of its arithmetic,
on memory sizes (no GPU work), and transfer_between_devices (multidev:78-83,
a stub in the reference) on the device."""
import random

import numpy as np
import pytest

import opencuda_cuda as oc


def reference_partition(mem, total_layers):
    """multidev:28-74: floor(total * mem_i / sum) for every device but the
    last, which takes the rest; an equal split when all report 0."""
    total = sum(mem)
    out, offset = [], 0
    for i, m in enumerate(mem):
        if i + 1 == len(mem):
            n = total_layers - offset
        elif total == 0:
            n = total_layers // len(mem)
        else:
            n = total_layers * m // total
        end = min(offset + n, total_layers)
        out.append((i, offset, end))
        offset = end
    return out


CASES = [
    ([24 << 30, 24 << 30], 40),           # RTX 4090 + RX 7900 XTX: 20 / 20
    ([183359 << 20] * 8, 61),             # eight B200s, remainder on the last
    ([16 << 30, 48 << 30], 40),           # 10 / 30
    ([0, 0, 0], 10),                      # no memory reported: 3 / 3 / 4
    ([8 << 30], 12),                      # one device takes all
    ([1, 1, 1, 1], 2),                    # fewer layers than devices
    ([0, 5], 7),                          # a zero-memory device among others
]


@pytest.mark.parametrize("mem,layers", CASES)
def test_partition_by_memory(mem, layers):
    got = oc.partition_layers_by_memory(mem, layers)
    assert got == reference_partition(mem, layers)
    assert got[-1][2] == layers and got[0][1] == 0
    assert all(a[2] == b[1] for a, b in zip(got, got[1:]))


def test_partition_random_against_restatement():
    rnd = random.Random(5)
    for _ in range(300):
        n = rnd.randint(1, 9)
        mem = [rnd.choice([0, rnd.randint(1, 1 << 40)]) for _ in range(n)]
        layers = rnd.randint(0, 200)
        assert oc.partition_layers_by_memory(mem, layers) == reference_partition(mem, layers)


def test_partition_rejects_empty_list():
    with pytest.raises(ValueError, match="no devices to partition across"):
        oc.partition_layers_by_memory([], 10)


@pytest.mark.gpu
def test_partition_and_transfer_on_devices():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    n = min(torch.cuda.device_count(), 2)
    devs = [oc.Device(i) for i in range(n)]
    try:
        mem = [d.info().total_memory for d in devs]
        assert oc.partition_layers(devs, 48) == reference_partition(mem, 48)
        payload = np.random.default_rng(7).integers(0, 255, size=(5 << 20) + 12, dtype=np.uint8)
        src = devs[0].alloc(payload.size)
        devs[0].memcpy_h2d(src, payload)
        for d in devs:  # the same device, then (with two GPUs) the peer over NVLink
            dst = d.alloc(payload.size)
            oc.transfer_between_devices(devs[0], src, d, dst, payload.size)
            back = np.zeros_like(payload)
            d.memcpy_d2h(back, dst)
            assert np.array_equal(back, payload)
            with pytest.raises(ValueError):
                oc.transfer_between_devices(devs[0], src, d, dst, payload.size + 1)
            d.free(dst)
        devs[0].free(src)
    finally:
        for d in devs:
            d.close()
