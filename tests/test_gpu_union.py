"""GPU parity of the union/compaction kernels (bit-exact) against the oracle
and the reference's own naive_sparsity_div outputs."""
import numpy as np
import pytest

from conftest import golden_union_cases

pytestmark = pytest.mark.gpu


def _to_dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("case", list(golden_union_cases()), ids=lambda c: c[0])
def test_spb_union_matches_reference_golden(spb, cuda, case):
    name, lab, counts, flat = case
    groups = lab.shape[0] // 8
    merge, act_cum, _ = spb.union(_to_dev(lab[:groups * 8], cuda), group=8)
    merge, act_cum = merge.cpu().numpy(), act_cum.cpu().numpy()
    per = np.diff(np.concatenate([[0], act_cum]))
    np.testing.assert_array_equal(per, counts)
    got = np.concatenate([merge[g, :per[g]] for g in range(groups)])
    np.testing.assert_array_equal(got, flat)


SHAPES = [(1, 32), (1, 11008), (3, 77), (8, 11008), (17, 1000), (64, 11008), (256, 4096), (32, 28672)]


@pytest.mark.parametrize("B,f", SHAPES)
@pytest.mark.parametrize("group", [0, 8])
def test_spb_union_vs_oracle(spb, cuda, oracle_mod, B, f, group):
    rng = np.random.default_rng(B * 100003 + f)
    lab = np.where(rng.random((B, f)) < 0.1, rng.random((B, f)), -rng.random((B, f))).astype(np.float32)
    lab[:, ::97] = np.nan
    G = B if group == 0 else group
    merge, act_cum, bits = spb.union(_to_dev(lab, cuda), group=group)
    m_ref, c_ref = oracle_mod.union(lab, G)
    np.testing.assert_array_equal(act_cum.cpu().numpy(), np.cumsum(c_ref))
    merge = merge.cpu().numpy()
    for s in range(len(c_ref)):
        np.testing.assert_array_equal(merge[s, :c_ref[s]], m_ref[s, :c_ref[s]])
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), oracle_mod.token_bits(lab))


@pytest.mark.parametrize("fill", [0.0, 1.0])
def test_spb_union_empty_and_full(spb, cuda, fill):
    lab = np.full((16, 4096), fill, np.float32)
    merge, act_cum, _ = spb.union(_to_dev(lab, cuda), group=0)
    n = int(act_cum.cpu()[0])
    assert n == (4096 if fill else 0)
    if fill:
        np.testing.assert_array_equal(merge.cpu().numpy()[0], np.arange(4096))


def test_dropin_get_idx_cuda(spb, cuda, oracle_mod):
    """get_idx_cuda through the reference's C++ signature: cumulative counts,
    per-group ascending lists, floor(B/8) groups."""
    import torch
    rng = np.random.default_rng(9)
    B, f = 44, 11008  # 5 full groups, 4 tokens ignored as in the reference
    lab = (rng.random((B, f)) < 0.08).astype(np.float32)
    groups = B // 8
    idx = _to_dev(lab, cuda)
    merge = torch.full((groups * f,), -7, dtype=torch.int32, device=cuda)
    act = torch.zeros(groups, dtype=torch.int32, device=cuda)
    fn = spb.dropin.fn("get_idx_cuda")
    fn(idx.data_ptr(), merge.data_ptr(), act.data_ptr(), B, f, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    m_ref, c_ref = oracle_mod.union(lab[:groups * 8], 8)
    np.testing.assert_array_equal(act.cpu().numpy(), np.cumsum(c_ref))
    merge = merge.cpu().numpy().reshape(groups, f)
    for g in range(groups):
        np.testing.assert_array_equal(merge[g, :c_ref[g]], m_ref[g, :c_ref[g]])
