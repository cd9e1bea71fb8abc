"""GPU parity of the position + timestamp embedding add (torch operator -> C ABI) against the golden
vectors of the reference's compiled operator: indices bit-exact, sums within one unit in the last
place of the element type (float32: 2e-6 absolute of O(1) values); the sorted index outputs must be
sorted and their permutations must map the per-token indices onto them."""
import os

import numpy as np
import pytest
import torch

import recir_b200  # noqa: F401
from oracle import embed_oracle as eo

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "embed_golden.npz"))
CASES = sorted({k.split("/")[0] for k in GOLD.files})
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
ULP = {"float32": 2e-6, "bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}


def unsort(sorted_vals, order):
    out = torch.empty_like(sorted_vals)
    out[order.long()] = sorted_vals
    return out


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("idx_dtype", [torch.int64, torch.int32])
def test_matches_reference_golden(name, idx_dtype):
    dt, tdt, c, inter, fn = (str(v) for v in GOLD[f"{name}/cfg"])
    lengths = GOLD[f"{name}/lengths"]
    tg = GOLD[f"{name}/targets"]
    off = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=idx_dtype, device="cuda")
    cu = lambda key, d=None: torch.as_tensor(GOLD[f"{name}/{key}"]).to(d).cuda() if d else torch.as_tensor(GOLD[f"{name}/{key}"]).cuda()  # noqa: E731
    y, sp, po, st, to = torch.ops.recir.b200_add_ts_pos_emb_fwd(
        cu("x", DT[dt]), off, cu("pos", DT[tdt]), cu("ts", DT[tdt]), cu("stamps"),
        torch.as_tensor(lengths).to(idx_dtype).cuda(), None if tg[0] < 0 else torch.as_tensor(tg).to(idx_dtype).cuda(),
        int(lengths.max()), int(c), inter == "1", fn)
    torch.cuda.synchronize()
    assert sp.dtype == torch.int32 and po.dtype == torch.int32
    assert (sp[1:] >= sp[:-1]).all() and (st[1:] >= st[:-1]).all()
    assert torch.equal(unsort(sp, po).cpu(), torch.as_tensor(GOLD[f"{name}/pos_idx"]))
    assert torch.equal(unsort(st, to).cpu(), torch.as_tensor(GOLD[f"{name}/ts_idx"]))
    want = GOLD[f"{name}/y"].astype(np.float64)
    tol = ULP[dt] * np.maximum(np.abs(want), 1.0 if dt == "float32" else 1e-3)
    assert (np.abs(y.float().cpu().numpy() - want) <= tol).all()


def test_benchmark_size_against_the_oracle():
    bt = recir_b200.workload.config1()
    g = torch.Generator().manual_seed(9)
    lengths = np.asarray(bt.lengths)
    b, t, cols = len(lengths), bt.total_tokens, 512
    x = torch.randn(t, cols, generator=g).to(torch.bfloat16)
    pos = torch.randn(2200, cols, generator=g).to(torch.bfloat16)
    ts = torch.randn(2049, cols, generator=g).to(torch.bfloat16)
    gaps = torch.exp(torch.rand(b, int(lengths.max()), generator=g) * 12.0).to(torch.int64)
    stamps = torch.cumsum(gaps, dim=1) + 1_600_000_000
    tg = bt.num_targets
    y, sp, po, st, to = torch.ops.recir.b200_add_ts_pos_emb_fwd(
        x.cuda(), bt.seq_offsets.cuda(), pos.cuda(), ts.cuda(), stamps.cuda(), torch.as_tensor(lengths).cuda(), tg.cuda(),
        int(lengths.max()), 2, False, "sqrt")
    torch.cuda.synchronize()
    ry, rp, rt = eo.add_ts_pos_emb(x.float().numpy(), bt.seq_offsets.numpy(), pos.float().numpy(), ts.float().numpy(),
                                   stamps.numpy(), lengths, tg.numpy(), 2, False, "sqrt", "bfloat16")
    assert np.array_equal(unsort(sp, po).cpu().numpy(), rp)
    assert np.array_equal(unsort(st, to).cpu().numpy(), rt)
    assert np.array_equal(y.float().cpu().numpy(), ry)  # sqrt is exactly rounded: bit-exact
