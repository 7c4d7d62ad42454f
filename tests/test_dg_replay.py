"""Slot-table parity of the device-gated cache on the CPU: this library's slot cache (tsb_test_dg_replay) against the
reference's own DgCore (oracle/_ref/libtsref.so) on the same configuration and trace, token by token: the uploaded
slot table and the counters must be identical, and with bytes moved every read through the table must find the
routed unit's bytes."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime, synth


def make_case(G=6, U=16, parts=(2048, 2048, 4096), R=4, D=1, B=4, Q=None, tokens=40, s=1.1, seed=7, n_pred=0,
              wb_defer=1, wb_on_d2h=1, uniform=False, rho=0.0, **kw):
    """A gated model of G layers x U units with R residents and D spare slots per layer (the C2 shape, scaled)."""
    top_k = B
    ids = synth.zipf_trace(tokens, G, U, top_k, s=s, seed=seed, uniform=uniform, rho=rho)
    order = []
    pop = synth.popularity_order(G, U, s=s, seed=seed)
    for g in range(G):
        order += [g * U + e for e in pop[g][:R]]
    P = G * U - len(order)
    Q = Q if Q is not None else D * G
    preds = None
    if n_pred:
        preds = synth.zipf_trace(tokens, G, U, n_pred, s=s, seed=seed + 1000)
    cfg = runtime.replay_config([U] * G, list(parts), persistent_slots=len(order) + D * G, bank_slots=B,
                                blocks=P + Q, spare_target=D * G, order=order, tokens=tokens, n_ids=top_k,
                                n_pred=n_pred, wb_defer=wb_defer, wb_on_d2h=wb_on_d2h, **kw)
    return cfg, ids, preds


CASES = {
    "c2_shape_deferred": dict(),
    "boundary_writebacks": dict(wb_defer=0),
    "deferred_on_demand_stream": dict(wb_on_d2h=0),
    "uniform_routes": dict(uniform=True),
    "correlated_top8": dict(G=5, U=32, R=8, D=2, B=8, rho=0.5, s=0.9),
    "predictions": dict(n_pred=2),
    "predictions_tight_budget": dict(n_pred=3, prefetch_per_layer=1, prefetch_per_token=4),
    "few_spare_blocks": dict(Q=2, D=3),
    "one_spare_slot": dict(G=4, U=8, R=2, D=1, B=2, Q=1),
    "zero_reserve_prefetch": dict(n_pred=2, prefetch_reserve=0),
    "small_credit": dict(wb_layer_bytes=1024, wb_max_outstanding=4096),
    "inclusive_share": dict(inclusive=5, Q=8),
    "inclusive_share_boundary_writebacks": dict(inclusive=20, Q=24, wb_defer=0, D=2),
    "inclusive_with_predictions": dict(inclusive=12, Q=16, n_pred=2),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_slot_tables_match_reference(ref, name):
    cfg, ids, preds = make_case(**CASES[name])
    t_ref, s_ref = oracle.ref_replay(cfg, ids, preds)
    t_new, s_new = runtime.replay(cfg, ids, preds)
    for t in range(cfg.tokens):
        assert np.array_equal(t_new[t], t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(s_new[t], s_ref[t]), "counters differ after token %d: %s vs %s" % (
            t, s_new[t].tolist(), s_ref[t].tolist())
    assert s_new[-1][2] > 0, "the case must exercise misses"


def test_bytes_through_the_table(ref):
    G, U, parts = 4, 12, (256, 512, 256)
    cfg, ids, _ = make_case(G=G, U=U, parts=parts, R=3, D=1, B=2, tokens=30)
    cfg.move_bytes = 1
    unit = sum(parts)
    src = np.random.default_rng(3).integers(0, 256, size=G * U * unit, dtype=np.uint8)
    _, _, r_new = runtime.replay(cfg, ids, src_units=src, want_reads=True)
    _, _, r_ref = oracle.ref_replay(cfg, ids, src_units=src, want_reads=True)
    assert np.array_equal(r_new, r_ref)
    orc = oracle.orc()
    for t in range(cfg.tokens):
        for g in range(G):
            for i, e in enumerate(ids[t, g]):
                k = g * U + int(e)
                want = orc.orc_checksum(src[k * unit:(k + 1) * unit].ctypes.data, unit)
                assert r_new[t, g, i] == want


def test_replay_rejects_bad_ids():
    from tierstream_b200 import abi
    cfg, ids, _ = make_case(G=2, U=4, R=1, D=1, B=2, tokens=2)
    ids = ids.copy()
    ids[1, 1, 0] = 9
    with pytest.raises(abi.TsError) as e:
        runtime.replay(cfg, ids)
    assert e.value.status == abi.SS_E_INVALID
