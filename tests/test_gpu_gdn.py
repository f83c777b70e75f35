"""GPU parity of the chunked GatedDeltaNet kernels (r97b_gdn_fwd / r97b_gdn_bwd) against the f64 oracle
of the reference's gdn_kkt_solve + gdn_chunk_scan pair, through the C ABI: ragged sequences with short
last chunks, grouped heads, initial and final states. Inputs are rounded to bf16 first so both sides see
the same numbers; tolerance is the north star's bf16 bar."""
import numpy as np
import pytest
import torch

from oracle import gdn as G
from r97training_b200.gdn import GdnPlan
from tests.gpu_util import assert_close_bf16, to_np

pytestmark = pytest.mark.gpu


def _bf16(x):
    return torch.from_numpy(np.asarray(x, np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("lens,H,Hg,states,decay", [((64,), 2, 2, False, 1.0), ((200, 64, 1, 130), 4, 2, True, 1.0),
                                                    ((512,), 4, 4, False, 1.0), ((300, 64), 4, 2, True, 40.0)])
def test_gdn_fwd_bwd_vs_oracle(cuda, lens, H, Hg, states, decay):
    """decay scales the per-token log decay: 40 drives e^{g_i - g_j} far past f32's range above the
    diagonal (where it must never be formed) and to zero below it."""
    d = G.synth_inputs(list(lens), H, Hg, seed=sum(lens) + H)
    d["g"] = d["g"] * decay
    q, k, v, do = (_bf16(d[n]) for n in ("q", "k", "v", "do"))
    # the oracle sees exactly the bf16 values the kernels read
    qn, kn, vn, don = (t.double().numpy() for t in (q, k, v, do))
    g = d["g"].astype(np.float32)
    beta = d["beta"].astype(np.float32)
    rs = np.random.RandomState(1)
    h0 = (rs.normal(size=(len(lens), H, 128, 128)) * 0.05).astype(np.float32) if states else None
    dht = (rs.normal(size=(len(lens), H, 128, 128)) * 0.01).astype(np.float32) if states else None
    ref = G.layer_fwd_bwd(qn, kn, vn, g.astype(np.float64), beta.astype(np.float64), d["cu"], don,
                          h0=None if h0 is None else h0.astype(np.float64),
                          dht=None if dht is None else dht.astype(np.float64))
    plan = GdnPlan(d["cu"], H, Hg, cuda)
    dev = lambda t: t.to(cuda).contiguous()
    h0d = None if h0 is None else torch.from_numpy(h0).to(cuda)
    o, ht, sv = plan.forward(dev(q), dev(k), dev(v), torch.from_numpy(g).to(cuda), torch.from_numpy(beta).to(cuda),
                             h0=h0d, want_ht=True)
    grads = plan.backward(sv, dev(do), dht=None if dht is None else torch.from_numpy(dht).to(cuda),
                          want_dh0=True)
    torch.cuda.synchronize()
    assert_close_bf16(to_np(sv["A"]), ref["A"], rel=1e-4, what="A")
    assert_close_bf16(to_np(o), ref["o"], what="o")
    assert_close_bf16(to_np(ht), ref["ht"], rel=2e-3, what="ht")
    for name in ("dq", "dk", "dv", "dbeta", "dg"):
        assert_close_bf16(to_np(grads[name]), ref[name], what=name)
    if states:
        assert_close_bf16(to_np(grads["dh0"]), ref["dh0"], rel=2e-3, what="dh0")
