"""Host logic of the prepared cross-attention context (CPU): the byte
dedupe of context rows (whole_layer.py:50-58 of the reference's optimized
package) and the compact rows it keeps."""
import torch

from wam_ops.whole_layer import context_groups, prepared_context


def pairwise_groups(context):
    """The reference's loop: one torch.equal per (row, root) pair."""
    bits = context.contiguous().view(torch.uint8)
    roots, rows = [], []
    for row in range(context.shape[0]):
        group = next((g for g, root in enumerate(roots) if torch.equal(bits[row], bits[root])), None)
        if group is None:
            group = len(roots)
            roots.append(row)
        rows.append(group)
    return rows, roots


def test_context_groups_match_pairwise_loop():
    g = torch.Generator().manual_seed(3)
    base = torch.randn(5, 7, 16, generator=g).bfloat16()
    for pick in ([0], [0, 0], [0, 1, 0, 2, 1], [3, 3, 3, 3], [0, 1, 2, 3, 4], [4, 0, 4, 1, 0, 1, 2]):
        ctx = base[pick]
        assert context_groups(ctx) == pairwise_groups(ctx), pick


def test_context_groups_compare_bytes():
    """Rows that differ only in the sign of zero (equal as numbers) stay apart;
    a one-bit difference in the last element splits a group."""
    a = torch.zeros(1, 4, 8, dtype=torch.bfloat16)
    b = a.clone()
    b[0, 0, 0] = -0.0
    c = a.clone()
    c.view(torch.int16)[0, -1, -1] = 1
    assert context_groups(torch.cat((a, b, a, c))) == ([0, 1, 0, 2], [0, 1, 3])


def test_prepared_context_compacts_duplicates():
    g = torch.Generator().manual_seed(4)
    base = torch.randn(2, 3, 8, generator=g).bfloat16()
    rows, roots, compact = prepared_context(base[[1, 0, 1, 1]])
    assert rows.tolist() == [0, 1, 0, 0] and roots.tolist() == [0, 1]
    assert torch.equal(compact, base[[1, 0]])
    rows, roots, compact = prepared_context(base)
    assert rows is None and roots is None and torch.equal(compact, base)
