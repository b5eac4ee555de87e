"""State images on the device: export, import into a fresh state, and both
states continue identically (verify logits bit for bit, MTP drafts too);
the image matches its documented layout; damaged images are refused."""
import numpy as np
import pytest

from inferq_b200 import image, synth
from inferq_b200._lib import IqError
from inferq_b200.model import Model, State

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(cuda):
    cfg = synth.mini_35b()
    return cfg, Model(cfg, list(synth.generate(cfg, seed=13)))


def test_imported_state_continues_bitwise(model):
    cfg, m = model
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, cfg.vocab_size, 21)
    a = State(m, 128)
    am, _, hid = a.forward(prompt, hidden=True)
    a.mtp_sync(0, None, prompt, hid)
    img = a.export_image()
    parsed = image.parse(img, cfg)
    assert parsed["position"] == len(prompt) and parsed["mtp_position"] == len(prompt)
    b = State(m, 128)
    b.forward(rng.integers(0, cfg.vocab_size, 5))  # unrelated history, replaced by the import
    b.import_image(img)
    assert b.position == a.position and b.mtp_position == a.mtp_position
    drafts = [int(am[-1]), 11, 7, 300]
    ra, la, _ = a.verify(drafts, logits=True)
    rb, lb, _ = b.verify(drafts, logits=True)
    assert ra == rb and np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    da = a.mtp_draft(int(ra[1]), hid[-1], 2, cfg.vocab_size)
    db = b.mtp_draft(int(rb[1]), hid[-1], 2, cfg.vocab_size)
    assert np.array_equal(da[0], db[0]) and np.array_equal(da[1].view(np.uint32), db[1].view(np.uint32))


def test_damaged_images_are_refused(model):
    cfg, m = model
    a = State(m, 64)
    a.forward([1, 2, 3])
    img = a.export_image()
    b = State(m, 64)
    with pytest.raises(IqError):
        b.import_image(img[:-4])
    bad = img.copy()
    bad[:8] = np.frombuffer(b"XXXXXXXX", np.uint8)
    with pytest.raises(IqError):
        b.import_image(bad)
    small = State(m, 2)  # too few positions for the image
    with pytest.raises(IqError):
        small.import_image(img)
