"""The committed .order files of the benchmark models (emufpga_b200/orders/):
each is what the library's default consumption order gives for its model,
names exactly the model's tensors (spm_order_check in both directions,
spm-order/src/order.rs:64-111), and walks the rotating region in the order a
decode step reads it."""
from pathlib import Path

import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from emufpga_b200.orders import make_orders as M
from tests.test_order_sweep import demands, parse

ORDERS = Path(M.__file__).resolve().parent


@pytest.mark.parametrize("name", sorted(M.MODELS))
def test_committed_order_is_the_default_order(name):
    assert (ORDERS / name).read_text() == M.order_text(M.MODELS[name])


@pytest.mark.parametrize("name", sorted(M.MODELS))
def test_committed_order_names_exactly_the_models_tensors(name):
    mini = M.miniature(configs.RECIPES[M.MODELS[name]])
    eb.order_check((ORDERS / name).read_text(), eb.synth_gguf(mini))


@pytest.mark.parametrize("name", sorted(M.MODELS))
def test_committed_order_is_the_step_order(name):
    shape = configs.RECIPES[M.MODELS[name]].shape
    rot, res = parse((ORDERS / name).read_text())
    assert rot == demands(shape)
    assert "token_embd.weight" in res
    if shape.moe:
        assert all(f"blk.{l}.exp_probs_b.bias" in res for l in range(shape.layers))
