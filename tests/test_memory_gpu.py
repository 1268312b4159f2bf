"""O(1) activation memory of reversible stages, measured on the device.

One GPU, one stage (embedding + blocks + head), BERT-Large width, 4 x 512 tokens per
micro-batch.  The memory a training step allocates on top of what lives between steps
(weights, gradients, Adam state, receive rings, scratch) must not grow with the number of
blocks for reversible stages; for standard stages (every block's activations kept until
its backward) it must.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _step_transient_bytes(layers: int, reversible: bool) -> int:
    from revpp.config import GlobalConfig
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger
    from revpp.utils.seed import set_seed

    dev = torch.device("cuda", 0)
    cfg = GlobalConfig(model="bert", reversible=reversible, num_hidden_layers=layers, hidden_size=1024,
                       num_attention_heads=16, max_position_embeddings=512, num_classes=2,
                       autocast_dtype=torch.bfloat16, batch_size=8, microbatch_size=4, num_microbatches=2, lr=1e-5)
    env = EnvContext(world_size=1, rank=0, local_rank=0, device=dev, proc_logger=build_logger("memtest", None),
                     node_logger=None, main_logger=None, pg=None, master_rank=0, num_stages=1, replicas=1)
    set_seed(0)
    tr = Trainer(cfg, env)
    batch = SyntheticBatches(cfg, 8, 1, seed=0).make(0)
    tr.train_step(batch)  # first step allocates the persistent scratch
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    tr.train_step(batch)
    torch.cuda.synchronize()
    transient = torch.cuda.max_memory_allocated() - base
    tr.close()
    del tr
    torch.cuda.empty_cache()
    return transient


def test_reversible_activation_memory_independent_of_blocks():
    t2 = _step_transient_bytes(2, True)
    t6 = _step_transient_bytes(6, True)
    assert t6 <= 1.05 * t2 + (16 << 20), (t2, t6)


def test_standard_activation_memory_grows_with_blocks():
    t2 = _step_transient_bytes(2, False)
    t6 = _step_transient_bytes(6, False)
    assert t6 > 1.5 * t2, (t2, t6)


@pytest.mark.parametrize("layers,reversible,mbs", [(2, True, 8), (4, True, 8), (2, True, 16), (2, False, 8)])
def test_memory_predictor_matches_measured_peak(layers, reversible, mbs):
    """The analytic predictor (used by the profiling experiment and the PaBER micro-batch
    search) is within 15 % of the measured peak of a single-stage training step."""
    from revpp.config import GlobalConfig
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.experiments.memory_predictor import predict_peak_bytes
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger
    from revpp.utils.seed import set_seed

    dev = torch.device("cuda", 0)
    torch.cuda.empty_cache()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    cfg = GlobalConfig(model="bert", reversible=reversible, num_hidden_layers=layers, hidden_size=1024,
                       num_attention_heads=16, max_position_embeddings=512, num_classes=2,
                       autocast_dtype=torch.bfloat16, batch_size=2 * mbs, microbatch_size=mbs, num_microbatches=2,
                       lr=1e-5)
    env = EnvContext(world_size=1, rank=0, local_rank=0, device=dev, proc_logger=build_logger("mempred", None),
                     node_logger=None, main_logger=None, pg=None, master_rank=0, num_stages=1, replicas=1)
    set_seed(0)
    tr = Trainer(cfg, env)
    batch = SyntheticBatches(cfg, 2 * mbs, 1, seed=0).make(0)
    for _ in range(2):
        tr.train_step(batch)
    torch.cuda.synchronize()
    measured = torch.cuda.max_memory_allocated() - base
    kind = "reversible" if reversible else "standard"
    predicted = predict_peak_bytes(cfg, 0, 1, kind)
    tr.close()
    del tr
    torch.cuda.empty_cache()
    assert abs(predicted - measured) <= 0.15 * measured, (predicted / 2**30, measured / 2**30)
