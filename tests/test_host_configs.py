"""The benchmark and parity presets have the shapes the baseline configs
name (CPU): configs[0] / [1] one 1536-wide block and its 30-layer stack over
1560 video + 32 action tokens, configs[2] the 5B-shape stack over an
880-token chunk (848 video + 32 action) with a 4-chunk history, configs[3]
4 candidate chunks of 32 action tokens against that history, and the bench
workload 8 such rollouts per GPU; 512 context tokens throughout."""
import pytest

from wam_ops import configs


@pytest.mark.parametrize("name,dim,heads,ffn,layers", [
    ("cfg0", 1536, 12, 8960, 1), ("cfg1", 1536, 12, 8960, 30),
    ("cfg2", 3072, 24, 14336, 30), ("cfg3", 3072, 24, 14336, 30), ("cfg4", 3072, 24, 14336, 30),
])
def test_preset_model_shapes(name, dim, heads, ffn, layers):
    c = configs.PRESETS[name]
    assert (c.dim, c.heads, c.ffn, c.layers) == (dim, heads, ffn, layers)
    assert c.dim == c.heads * 128
    assert c.context == 512


def test_preset_token_counts():
    P = configs.PRESETS
    assert P["cfg0"].tokens == P["cfg1"].tokens == 1560 + 32
    assert P["cfg2"].tokens == P["cfg4"].tokens == 848 + 32
    assert P["cfg2"].history_chunks * P["cfg2"].tokens == 3520
    assert P["cfg3"].candidates == 4 and P["cfg3"].history_chunks * P["cfg2"].tokens == 3520
    assert P["cfg4"].batch == 8
