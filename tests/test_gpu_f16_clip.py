"""f16 range of the activations: a forward that clips an f16 activation must
say so (WC_W_F16_CLIPPED, an F16ClipWarning in Python) and still deliver its
outputs; a normal checkpoint must not trigger it.

The clipping checkpoint is the tiny model with its feed-forward RMSNorm
weights at 400: the gated-GELU inputs then have a standard deviation of
about 130, so gelu(x W0) * (x W1) runs far past 65504.  The f32 oracle has no
such limit, and the test records how far the clipped result moves from it."""
import warnings

import numpy as np
import pytest

from oracle import oracle as O
from witchcraft_b200._lib import F16ClipWarning
from witchcraft_b200.synth import T5Config, make_synthetic_model
from witchcraft_b200.t5cuda import T5EncoderModel

from gpu_util import cosine_rows

pytestmark = pytest.mark.gpu


def _cfg():
    return T5Config(vocab_size=512, d_model=256, d_ff=512, num_heads=4, num_layers=2)


@pytest.mark.parametrize("B,L", [(2, 16), (3, 100), (8, 128)])  # small-M GEMV, 1-SM and 2-SM GEMM paths
def test_clipping_is_reported(B, L):
    m = make_synthetic_model(_cfg(), seed=3, ff_norm_weight=400.0)
    enc = T5EncoderModel(m.gguf, m.config.to_json(), 0)
    try:
        ids = np.random.default_rng(B).integers(3, 512, (B, L)).astype(np.uint32)
        with warnings.catch_warnings(record=True) as w:
            warnings.simplefilter("always")
            out = enc.forward(ids)
        assert any(issubclass(x.category, F16ClipWarning) for x in w), [str(x.message) for x in w]
        assert np.isfinite(out).all()
        cos = cosine_rows(out, O.OracleEncoder(m).encode(ids))
        print(f"B={B} L={L}: cosine vs f32 oracle with clipping min {cos.min():.4f} median {np.median(cos):.4f}")
        # the next call on normal inputs of a normal model starts clean
    finally:
        enc.close()


def test_normal_model_does_not_report_clipping(xtr_model):
    enc = T5EncoderModel(xtr_model.gguf, xtr_model.config.to_json(), 0)
    try:
        for B, L in ((1, 32), (4, 200), (16, 128)):
            ids = np.random.default_rng(L).integers(3, 32128, (B, L)).astype(np.uint32)
            with warnings.catch_warnings():
                warnings.simplefilter("error", F16ClipWarning)
                enc.forward(ids)
    finally:
        enc.close()
