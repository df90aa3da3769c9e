"""Load balance of the tensor-core kernel's persistent walk (CPU only).

Restates, in numpy, the item numbering (tc_item), the snake walk over the grid (tc_item_index) and
the BERT work order (bert_item_order: items sorted by key-tile count, most first) of
ligguf_b200/csrc/flash_tc.cuh, and checks the per-CTA key-tile loads that the kernel comments quote:
BERT lengths U[16, 512] give the busiest CTA 14-39 % above the mean in the natural order and 1-4 %
when sorted; causal prefill (heaviest first by numbering) about 5 %.  The ordering inside one cost
is arbitrary in the kernel (shared-memory atomics) and does not change these loads."""
import numpy as np

SMS = 148
ROWS = KEYS = 128


def snake_loads(costs, grid=SMS):
    """Key tiles per CTA when CTA c takes walk positions w * grid + (c, or grid - 1 - c on odd w)."""
    load = np.zeros(grid)
    n = len(costs)
    for w in range((n + grid - 1) // grid):
        for c in range(grid):
            p = w * grid + ((grid - 1 - c) if w & 1 else c)
            if p < n:
                load[c] += costs[p]
    return load


def bert_costs(lens, n_heads, max_len):
    """Key tiles of each item in tc_item numbering: head fastest, then query tile from the last, then batch."""
    n_qt = (max_len + ROWS - 1) // ROWS
    costs = []
    for b, ln in enumerate(lens):
        ln = min(ln, max_len)
        for y in range(n_qt):
            r0 = (n_qt - 1 - y) * ROWS
            c = 0 if r0 >= ln else (ln + KEYS - 1) // KEYS
            costs += [c] * n_heads
    return np.array(costs, float)


def counting_sort_desc(costs):
    order = np.argsort(-costs, kind="stable")
    assert sorted(order.tolist()) == list(range(len(costs)))  # a permutation
    return costs[order]


def excess(load):
    return load.max() / load.mean() - 1.0


def test_bert_sorted_walk_is_balanced():
    rng = np.random.default_rng(0)
    nat, srt = [], []
    for _ in range(8):
        lens = rng.integers(16, 513, 64)
        costs = bert_costs(lens, 12, 512)
        nat.append(excess(snake_loads(costs)))
        srt.append(excess(snake_loads(counting_sort_desc(costs))))
    assert min(nat) > 0.10, nat
    assert max(srt) < 0.05, srt


def test_prefill_heaviest_first_numbering_is_near_balanced():
    heads, n_qt = 32, 2048 // ROWS
    costs = np.array([n_qt - ((i // heads) % n_qt) for i in range(heads * n_qt)], float)
    assert np.all(np.diff(costs) <= 0)  # already heaviest first
    assert excess(snake_loads(costs)) < 0.06
