"""Rank layout and GPU placement rules (no GPU needed: the device count is a parameter)."""
import pytest

from trenowanie_generatora_obrazkow_b200.parallel.placement import RankLayout, local_device


def _order(layout, n_dev=8, **kw):
    return [local_device(i, n_dev, layout, **kw) for i in range(layout.world_all)]


def test_layout_roles_in_order():
    lay = RankLayout(8, actors=1, teachers=1, lm_servers=1, vae_servers=1)
    assert [lay.role(r) for r in range(8)] == ["learner"] * 4 + ["actor", "teacher", "lm", "vae"]
    assert lay.lm_server_of(3) == 6
    lay2 = RankLayout(6, lm_servers=2)
    assert lay2.lm_clients(4, pp=2) == [0] and lay2.lm_clients(5, pp=2) == [2]


def test_default_and_skip():
    lay = RankLayout(8)
    assert _order(lay) == list(range(8))
    lay6 = RankLayout(6)
    assert _order(lay6, skip_gpus=[1, 4]) == [0, 2, 3, 5, 6, 7]
    with pytest.raises(ValueError):
        local_device(0, 8, RankLayout(7), skip_gpus=[1, 4])


def test_lm_and_vae_gpus_go_last():
    lay = RankLayout(8, lm_servers=1, vae_servers=1)
    assert _order(lay, lm_gpu=2, vae_gpu=5) == [0, 1, 3, 4, 6, 7, 2, 5]
    with pytest.raises(ValueError):
        _order(lay, lm_gpu=3, vae_gpu=3)


def test_actor_and_teacher_gpus():
    lay = RankLayout(8, actors=2, teachers=1, lm_servers=1)
    order = _order(lay, lm_gpu=0, actor_gpus=[6, 7], teacher_gpu=5)
    # learners 0-3, actors 4-5, teacher 6, LM server 7
    assert order == [1, 2, 3, 4, 6, 7, 5, 0]
    lay2 = RankLayout(8, actors=2, lm_servers=1)
    assert _order(lay2, lm_gpu=7, actor_gpus=[0, 1]) == [2, 3, 4, 5, 6, 0, 1, 7]
    with pytest.raises(ValueError):
        _order(lay2, lm_gpu=7, actor_gpus=[7, 1])
