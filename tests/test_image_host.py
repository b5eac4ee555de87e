"""State-image layout on CPU: header, size formula and parsing of a
hand-built image for the tiny and the 35B-shaped configs."""
import numpy as np
import pytest

from inferq_b200 import image, synth


def _build(cfg, pos, mpos, rng):
    sh = image.shapes(cfg)
    h = np.zeros(1, image.HEADER)
    h["magic"], h["version"], h["layers"] = image.MAGIC, 1, cfg.num_hidden_layers
    h["position"], h["mtp_position"], h["has_mtp"] = pos, mpos, int(cfg.mtp_num_hidden_layers > 0)
    for k, v in sh.items():
        h[k] = v
    n = (image.image_bytes(cfg, pos, mpos) - image.HEADER.itemsize) // 4
    body = rng.standard_normal(n).astype(np.float32)
    return h.tobytes() + body.tobytes(), body


@pytest.mark.parametrize("make", [synth.tiny, synth.mini_35b, synth.qwen36_35b])
def test_image_round_trips_through_the_parser(make):
    cfg = make()
    rng = np.random.default_rng(0)
    buf, body = _build(cfg, 7, 5 if cfg.mtp_num_hidden_layers else 0, rng)
    out = image.parse(buf, cfg)
    assert out["position"] == 7
    flat = []
    for lay in out["layers"]:
        flat += [v.ravel() for v in lay.values()]
    if "mtp" in out:
        flat += [out["mtp"]["keys"], out["mtp"]["values"]]
    assert np.array_equal(np.concatenate(flat), body)


def test_image_rejects_truncation_and_foreign_shapes():
    cfg = synth.mini_35b()
    buf, _ = _build(cfg, 3, 2, np.random.default_rng(1))
    with pytest.raises(ValueError):
        image.parse(buf[:-4], cfg)
    with pytest.raises(ValueError):
        image.parse(b"NOTANIMG" + buf[8:], cfg)
    with pytest.raises(ValueError):
        image.parse(buf, synth.tiny())


@pytest.mark.parametrize("make", [synth.tiny, synth.mini_35b])
def test_build_is_the_inverse_of_parse(make):
    cfg = make()
    buf, _ = _build(cfg, 9, 4 if cfg.mtp_num_hidden_layers else 0, np.random.default_rng(2))
    again = image.build(cfg, image.parse(buf, cfg))
    assert again.tobytes() == buf


def test_oracle_state_image_round_trip():
    """The oracle's import/export of the library's image layout: an oracle
    state exported and imported into a fresh state continues identically."""
    import oracle
    cfg = synth.tiny()
    tensors = list(synth.generate(cfg, seed=4))
    om = oracle.OracleModel(cfg, tensors)
    a = om.state(64)
    a.forward([5, 9, 400])
    img = a.export_image()
    parsed = image.parse(img, cfg)
    assert parsed["position"] == 3
    assert np.any(parsed["layers"][0]["recurrent"] != 0) and np.any(parsed["layers"][3]["keys"] != 0)
    b = om.state(64)
    b.forward([1])
    b.import_image(img)
    assert b.position == 3
    la, _, _ = a.forward([77, 78])
    lb, _, _ = b.forward([77, 78])
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


def test_oracle_rollback_restores_the_committed_rows():
    """The oracle's verification snapshots: a 4-row pass rolled back to 2
    rows continues exactly like a 2-row pass (DeltaNet state from the
    snapshot, KV truncated by the position)."""
    import oracle
    cfg = synth.tiny()
    om = oracle.OracleModel(cfg, list(synth.generate(cfg, seed=6)))
    a, b = om.state(64), om.state(64)
    a.enable_snapshots(4)
    for st in (a, b):
        st.forward([3, 4, 5])
    a.forward([7, 8, 9, 10])
    a.rollback(2)
    b.forward([7, 8])
    assert a.position == b.position == 5
    la, _, _ = a.forward([11])
    lb, _, _ = b.forward([11])
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
