"""Generate tests/golden/formats.npz with gguf-py 0.19.0 as the decoder.

The reference decodes GGUF blocks with candle-core 0.11.0 (unvendored); gguf-py
implements the same published GGML block formats and its Q8_0 quantizer is
documented as bit-exact with ggml-quants.c, which candle's from_float mirrors.
Run from the repo root:  python tests/golden/make_golden.py
"""
from pathlib import Path
import sys

import numpy as np
import torch
from gguf import GGMLQuantizationType as T
from gguf import quants as gq

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from inferq_b200 import quants as Q  # noqa: E402

out = {}
torch.manual_seed(1234)
for dt, gt, cols in [(Q.Q4_K, T.Q4_K, 512), (Q.Q5_K, T.Q5_K, 512), (Q.Q6_K, T.Q6_K, 512),
                     (Q.Q8_0, T.Q8_0, 256)]:
    x = torch.randn(6, cols) * 0.02
    x[0, :7] = 0.0  # a partly flat region
    x[1] *= 40.0    # a large-magnitude row
    blocks = Q.encode(x, dt).numpy()
    out[f"{Q.NAMES[dt]}_bytes"] = blocks
    out[f"{Q.NAMES[dt]}_f32"] = gq.dequantize(blocks, gt).reshape(6, cols).astype(np.float32)
# Q8_0 activation quantization: gguf-py quantize_blocks (bit-exact with ggml).
act = (np.random.default_rng(7).standard_normal((3, 256)) * np.array([[0.01], [1.0], [30.0]])).astype(np.float32)
act[2, 40:72] = 0.0
out["act_f32"] = act
out["act_q8_0"] = gq.quantize(act, T.Q8_0)
np.savez_compressed(Path(__file__).with_name("formats.npz"), **out)
print("wrote", sum(v.nbytes for v in out.values()), "bytes")
