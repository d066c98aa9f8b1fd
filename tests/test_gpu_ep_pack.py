"""GPU, one device: the expert-parallel combine-row packing and the packed
combine against their CPU stand-ins (bit-exact: same power of two, same
round-to-nearest fp16 conversion, same fp32 summation order)."""
import pytest
import torch

from gemms_b200 import ep as EP
from tests.ep_fakes import CpuEpKernels

pytestmark = pytest.mark.gpu


def _rows():
    g = torch.Generator().manual_seed(1)
    mags = torch.tensor([1e-30, 1e-3, 1.0, 3e4, 1e8, 0.0, 2.0 ** 15, 0.5])
    return torch.randn(len(mags), 7168, generator=g) * mags.unsqueeze(1)


def test_pack_back_matches_cpu():
    rows = _rows()
    got = EP.CudaEpKernels().pack_back(rows.cuda()).cpu()
    want = CpuEpKernels(1, 1, 1).pack_back(rows)
    assert got.shape == want.shape
    H = rows.shape[1]
    assert torch.equal(got[:, :2 * H + 4], want[:, :2 * H + 4])


def test_packed_combine_matches_cpu():
    T, H, world = 33, 7168, 4
    g = torch.Generator().manual_seed(2)
    acc = torch.randn(T, H, generator=g) * 1e-3
    send_row_of = torch.full((T, world), -1, dtype=torch.int32)
    n = 0
    for t in range(T):
        for d in range(world):
            if (t + d) % 3 != 0:
                send_row_of[t, d] = n
                n += 1
    rows = torch.randn(n, H, generator=g) * 1e-3
    Kc, Kg = CpuEpKernels(1, 1, 1), EP.CudaEpKernels()
    packed = Kc.pack_back(rows)
    want = Kc.combine(acc, packed, send_row_of, world)
    got = Kg.combine(acc.cuda(), packed.cuda(), send_row_of.cuda(), world).cpu()
    # both sum acc + rows in destination order in fp32 and round once to bf16;
    # the GPU uses fma(h, 2^e, s), exact like the CPU's h * 2^e + s
    assert torch.equal(got, want)
