"""``torch.ops.flashdec.*`` inside ``torch.compile(fullgraph=True)``: a
compiled function that scales q, decodes through the custom operators and
post-processes the output gives the same bits as the same steps run eagerly
through the public functions (the operators run the same library launch)."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.golden import cases  # noqa: E402
from tests.helpers import to_dev  # noqa: E402

pytestmark = pytest.mark.gpu


def test_custom_ops_compile_fullgraph_and_match_eager():
    import flashdec_b200
    import flashdec_b200.ops  # noqa: F401

    c = cases.make_attn_case("split_257_193")
    q = to_dev(c["q"], "bfloat16")
    k, v = to_dev(c["k_cache"], "bfloat16"), to_dev(c["v_cache"], "bfloat16")
    bt, sl = to_dev(c["block_tables"]), to_dev(c["seq_lens"])

    def model(q, k, v, bt, sl, out):
        x = q * 2.0
        y = torch.ops.flashdec.decode(x, k, v, bt, sl)
        torch.ops.flashdec.decode_into(x, k, v, bt, sl, out)
        return y + 1.0, out * 3.0

    compiled = torch.compile(model, fullgraph=True, backend="aot_eager")
    out_c = torch.empty_like(q)
    y_c, o_c = compiled(q, k, v, bt, sl, out_c)

    x = q * 2.0
    y_e = flashdec_b200.decode(x, k, v, bt, sl) + 1.0
    out_e = torch.empty_like(q)
    flashdec_b200.paged_decode_attention_into(x, k, v, bt, sl, out_e)
    torch.cuda.synchronize()
    assert torch.equal(y_c, y_e)
    assert torch.equal(out_c, out_e)  # the mutated argument holds the decode
    assert torch.equal(o_c, out_e * 3.0)
    assert np.isfinite(y_c.float().cpu().numpy()).all()
