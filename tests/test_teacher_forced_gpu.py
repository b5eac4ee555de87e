"""Teacher-forced parity: every row of the device pass against the CPU oracle
(the reference's fp32 arithmetic in its own accumulation order), each row
started from the exact state the device holds.

Each step exports the device state (iq_state_export), imports it into the
oracle, advances both by one token and compares logits, the final
normalized hidden row and the state after the step.  Contexts cover one and
many 32-position attention chunks (positions 0, 31, 32, 33, 1023, 3071 and
the last position of a 4096-position state), starting from a seeded random
state image (random KV rows, conv history and recurrent state) so that long
contexts cost no prefill.

What is held, and why.  On these seeded random-init checkpoints a change at
the level of one f32 rounding anywhere in a row (another valid summation
order, one ulp on a norm output) flips some quantized activation by one
step, and the small residual stream amplifies that into logit changes of
0.01-0.15.  The oracle shows this against itself: run from the same state
in its alternative GEMV accumulation order, or with every RMSNorm output
moved by one ulp (two patterns), it lands more than 2e-2 away from itself on about a third
of the rows at 35B widths (the reference's own build-to-build differences,
AVX2 versus scalar summation, are of this kind).  So:

* strict, every row: the state a layer writes (its KV row, DeltaNet conv and
  recurrent state) within 2e-2 of the oracle's (measured: ~1e-5; a
  one-layer model, so no earlier layer feeds a flipped activation in);
* strict, every row: greedy tokens agree wherever the oracle's top-2 margin
  exceeds twice the tolerance;
* per configuration, over all rows, the device is held to the spread of
  the oracle's own variants (each one more valid implementation): median
  logit error within rounding (1e-4) or twice the variants' median gap; rows
  beyond 2e-2 no more frequent than for one variant (two binomial standard
  deviations of allowance); the largest error within twice the largest
  variant gap plus the tolerance.  Every device row beyond the tolerance is printed
  with the variants' largest gap on that row.
"""
import numpy as np
import pytest

import oracle
from inferq_b200 import image, synth
from inferq_b200.model import Model, State

pytestmark = pytest.mark.gpu

TOL = 2e-2
POSITIONS = (0, 31, 32, 33, 1023, 3071, 4095)
MAX_POS = 4096


def _35b_widths():
    c = synth.qwen36_35b()
    c.name = "qwen3.6-35b-widths-4-layers"
    c.num_hidden_layers = 4
    return c


def _80b_widths():
    c = synth.coder_next_80b()
    c.name = "coder-next-80b-widths-4-layers"
    c.num_hidden_layers = 4
    return c


CASES = {"tiny": synth.tiny, "mini_35b": synth.mini_35b, "35b_widths": _35b_widths, "80b_widths": _80b_widths}


@pytest.fixture(scope="module", params=list(CASES))
def pair(request, cuda):
    cfg = CASES[request.param]()
    cfg.max_position_embeddings = max(cfg.max_position_embeddings, MAX_POS)
    big = cfg.hidden_size >= 2048
    tensors = list(synth.generate(cfg, seed=17, device="cuda" if big else "cpu"))
    model = Model(cfg, tensors)
    om = oracle.OracleModel(cfg, tensors)
    yield cfg, model, om
    del model, om


def random_image(cfg, position, rng):
    """A state image at `position`: seeded KV rows, conv history and
    recurrent state of plausible magnitudes (all zeros at position 0, the
    true fresh state)."""
    sh = image.shapes(cfg)
    zero = position == 0
    layers = []
    for l in range(cfg.num_hidden_layers):
        if cfg.layer_is_full(l):
            layers.append({"keys": rng.standard_normal((position, sh["kv_dim"]), np.float32),
                           "values": rng.standard_normal((position, sh["kv_dim"]), np.float32)})
        else:
            conv = np.zeros((sh["conv_dim"], sh["conv_taps"]), np.float32)
            rec = np.zeros(sh["rec_size"], np.float32)
            if not zero:
                conv = rng.standard_normal(conv.shape, np.float32)
                rec = (0.05 * rng.standard_normal(rec.shape)).astype(np.float32)
            layers.append({"conv": conv, "recurrent": rec})
    parts = {"position": position, "mtp_position": position if cfg.mtp_num_hidden_layers else 0, "layers": layers}
    if cfg.mtp_num_hidden_layers:
        parts["mtp"] = {"keys": rng.standard_normal((position, sh["kv_dim"]), np.float32),
                        "values": rng.standard_normal((position, sh["kv_dim"]), np.float32)}
    return image.build(cfg, parts)


def _state_error(cfg, dev_img, ora_img, position):
    """Max abs difference of the two states: the KV row written at
    `position`, the DeltaNet conv and recurrent state."""
    a, b = image.parse(dev_img, cfg), image.parse(ora_img, cfg)
    err = 0.0
    for la, lb in zip(a["layers"], b["layers"]):
        if "keys" in la:
            for k in ("keys", "values"):
                err = max(err, float(np.abs(la[k][position] - lb[k][position]).max()))
                # rows before the step are the imported ones on both sides
                assert np.array_equal(la[k][:position], lb[k][:position])
        else:
            for k in ("conv", "recurrent"):
                err = max(err, float(np.abs(la[k] - lb[k]).max()))
    return err


def _margin(v):
    top2 = np.sort(v)[-2:]
    return float(top2[1] - top2[0])


VARIANTS = ((1, 0), (0, 1), (1, 1), (0, 2), (1, 2))  # (GEMV order, norm perturbation) besides the reference (0, 0)


def _oracle_row(ost, img, tok, order, perturb):
    ost.import_image(img)
    oracle.set_gemv_order(order)
    oracle.set_perturb(perturb)
    try:
        return ost.forward([int(tok)], hidden=True)
    finally:
        oracle.set_gemv_order(0)
        oracle.set_perturb(0)


def _run_rows(cfg, model, om, position, steps, rng, variants=VARIANTS):
    """Teacher-forced rows from a random image at `position`: per step the
    device's errors against the reference-order oracle and the oracle's own
    gap under rounding-level variants."""
    tokens = rng.integers(0, cfg.vocab_size, steps)
    st, ost = State(model, MAX_POS), om.state(MAX_POS)
    st.import_image(random_image(cfg, position, rng))
    out = []
    for i, tok in enumerate(tokens):
        img = st.export_image()
        am, lg, hd = st.forward([int(tok)], logits=True, hidden=True)
        olg, ohd, _ = _oracle_row(ost, img, tok, 0, 0)
        row = {"position": position + i, "argmax": int(am[0]), "ref_argmax": oracle.argmax(olg[0]),
               "margin": _margin(olg[0]), "logits": float(np.abs(lg[0] - olg[0]).max()),
               "hidden": float(np.abs(hd[0] - ohd[0]).max()),
               "state": _state_error(cfg, st.export_image(), ost.export_image(), position + i)}
        row["gaps"] = []
        for order, perturb in variants:
            vlg, _, _ = _oracle_row(ost, img, tok, order, perturb)
            row["gaps"].append(float(np.abs(vlg[0] - olg[0]).max()))
        out.append(row)
    return out


def _check_rows(name, rows, strict_state):
    """The device is one more valid implementation of the reference
    arithmetic; hold it to the spread of the oracle's own rounding-level
    variants (each a valid alternative implementation), row by row."""
    e = np.array([r["logits"] for r in rows])
    g = np.array([r["gaps"] for r in rows])  # [row][variant]
    n_dev = int((e > TOL).sum())
    n_var = int((g > TOL).sum(axis=0).max())
    over = [(r["position"], round(r["logits"], 4), round(max(r["gaps"]), 4)) for r in rows if r["logits"] > TOL]
    print(f"{name}: rows {len(rows)}, median logit error {np.median(e):.2e} (oracle variants "
          f"{np.median(g, axis=0).max():.2e}), max {e.max():.4f} (variants {g.max():.4f}); rows beyond TOL: device "
          f"{n_dev}, most of one oracle variant {n_var}; device rows beyond TOL (position, device error, largest "
          f"variant gap on that row) {over}; max state error {max(r['state'] for r in rows):.2e}")
    if strict_state:
        assert max(r["state"] for r in rows) <= TOL
    for r in rows:
        if r["argmax"] != r["ref_argmax"]:
            assert r["margin"] <= 2 * TOL, (r["position"], r["margin"])
    # typical row: rounding-level agreement, or no worse than the variants' typical gap
    assert np.median(e) <= max(1e-4, 2 * np.median(g, axis=0).max())
    # rows beyond the tolerance: no more frequent than for one oracle variant
    # (binomial allowance of two standard deviations)
    assert n_dev <= n_var + 2 * np.sqrt(n_var + 1)
    # size: the same order as the variants' largest gap
    assert e.max() <= 2 * g.max() + TOL


def _one_layer(cfg, kind):
    c = synth.Config(**{f.name: getattr(cfg, f.name) for f in __import__("dataclasses").fields(cfg)})
    c.name = f"{cfg.name}-{kind}-layer"
    c.num_hidden_layers = 1
    c.full_attention_interval = 1 if kind == "attention" else 4
    c.mtp_num_hidden_layers = 0
    return c


@pytest.fixture(scope="module", params=[(n, k) for n in CASES for k in ("deltanet", "attention")],
                ids=lambda p: f"{p[0]}-{p[1]}")
def layer_pair(request, cuda):
    name, kind = request.param
    cfg = _one_layer(CASES[name](), kind)
    cfg.max_position_embeddings = max(cfg.max_position_embeddings, MAX_POS)
    big = cfg.hidden_size >= 2048
    tensors = list(synth.generate(cfg, seed=23, device="cuda" if big else "cpu"))
    model = Model(cfg, tensors)
    om = oracle.OracleModel(cfg, tensors)
    yield cfg, model, om
    del model, om


def _all_rows(cfg, model, om, seed):
    rows = []
    for position in POSITIONS:
        rows += _run_rows(cfg, model, om, position, min(4, MAX_POS - position), np.random.default_rng(position + seed))
    return rows


def test_layer_rows_match_the_oracle_teacher_forced(layer_pair):
    """One decoder layer (DeltaNet or gated attention, then the MoE block)
    plus the final norm and LM head, at every listed context."""
    cfg, model, om = layer_pair
    _check_rows(cfg.name, _all_rows(cfg, model, om, 3), strict_state=True)


def test_rows_match_the_oracle_teacher_forced(pair):
    """The whole model (four layers), at every listed context."""
    cfg, model, om = pair
    _check_rows(cfg.name, _all_rows(cfg, model, om, 7), strict_state=False)


@pytest.mark.parametrize("position", (0, 33, 3071))
def test_mtp_draft_matches_the_oracle_teacher_forced(pair, position):
    cfg, model, om = pair
    if not cfg.mtp_num_hidden_layers:
        pytest.skip("no MTP block")
    rng = np.random.default_rng(position + 99)
    st, ost = State(model, MAX_POS), om.state(MAX_POS)
    st.import_image(random_image(cfg, position, rng))
    ost.import_image(st.export_image())
    hidden = rng.standard_normal(cfg.hidden_size).astype(np.float32)
    seed = int(rng.integers(0, cfg.vocab_size))
    vocab = min(cfg.vocab_size, 32768)
    tok, prob, margin, _ = st.mtp_draft(seed, hidden, 1, vocab)
    lg, _ = ost.mtp(seed, hidden, vocab)
    top = oracle.argmax(lg)
    p = 1.0 / np.sum(np.exp((lg - lg[top]).astype(np.float64)))
    assert abs(float(margin[0]) - _margin(lg)) <= TOL
    assert abs(float(prob[0]) - p) <= 2e-2 * p
    if _margin(lg) > 2 * TOL:
        assert int(tok[0]) == top
