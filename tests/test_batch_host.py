"""Host side of batched union decode (leanstream_b200/batch.py) on CPU:
union_plan's union, ExecDesc rows and per-token masks, slot and staging
mapping, argument errors; BatchMLP's argument checks, which the C ABI
answers before any CUDA call (no compute is launched here)."""
import errno

import numpy as np
import pytest


def test_union_plan_rows_and_masks():
    from leanstream_b200 import _native as N
    from leanstream_b200.batch import union_plan

    sets = [[5, 1, 9], [9, 12], [1], [40, 5, 3]]
    union, rows, mask = union_plan(sets)
    assert union.tolist() == [1, 3, 5, 9, 12, 40]
    assert rows.dtype == np.uint32 and rows.shape == (6, 5)
    assert rows[:, 0].tolist() == union.tolist()
    assert rows[:, 1].tolist() == union.tolist() and rows[:, 2].tolist() == union.tolist()
    assert rows[:, 3].tolist() == list(range(6)) and not rows[:, 4].any()
    assert mask.dtype == np.uint8 and mask.shape == (4, 6)
    for t, s in enumerate(sets):
        assert union[mask[t] == 1].tolist() == sorted(set(s))
    # slot / physical maps and streamed groups
    slots = np.arange(64)[::-1].copy()
    phys = (np.arange(64) * 3) % 64
    union, rows, _ = union_plan(sets, cache_slots=slots, physical=phys, staging={9: 2, 40: 7})
    assert rows[:, 1].tolist() == [int(phys[g]) for g in union]
    expect_slot = [int(slots[g]) if g not in (9, 40) else {9: 2, 40: 7}[g] for g in union]
    assert rows[:, 2].tolist() == expect_slot
    assert rows[:, 4].tolist() == [N.SOURCE_STAGING if g in (9, 40) else N.SOURCE_CACHE for g in union]


def test_union_plan_edges():
    from leanstream_b200.batch import union_plan

    union, rows, mask = union_plan([[], []])
    assert union.size == 0 and rows.shape == (0, 5) and mask.shape == (2, 0)
    union, rows, mask = union_plan([[3, 3, 3]])  # duplicates collapse
    assert union.tolist() == [3] and mask.tolist() == [[1]]
    with pytest.raises(ValueError):
        union_plan([])
    with pytest.raises(ValueError):
        union_plan([[1]] * 9)
    with pytest.raises(ValueError):
        union_plan([[1, -2]])


def test_batch_mlp_arguments_refused_on_host(native_lib):
    from leanstream_b200.batch import BatchMLP

    need = native_lib.ls_b200_batch_scratch_bytes(1024, 64, 12)
    with pytest.raises(ValueError):
        BatchMLP(1024, 64, 12, scratch=(1 << 25, need - 1))
    mlp = BatchMLP(1024, 64, 12, scratch=(1 << 25, need))
    good = dict(x=1 << 20, output=1 << 21, cache=1 << 22, scales=1 << 23, union_descs=1 << 24, union_count=12,
                tokens=8)
    with pytest.raises(ValueError):
        mlp.run(stream=0, **{**good, "union_count": 13})  # larger than the scratch was sized for
    for key, bad in [("tokens", 9), ("tokens", 0), ("x", None), ("x", (1 << 20) + 2), ("scales", (1 << 23) + 1),
                     ("hidden_out", 1 << 26)]:
        with pytest.raises(RuntimeError, match=errno.errorcode[errno.EINVAL]):
            mlp.run(stream=0, **{**good, key: bad})
    bad_geo = BatchMLP(1000, 64, 12, scratch=(1 << 25, 1 << 30))
    with pytest.raises(RuntimeError, match=errno.errorcode[errno.EINVAL]):
        bad_geo.run(stream=0, **good)
