"""Checkpoints written by the reference's own stage modules load into this framework's
stages strictly.

A subprocess builds the reference's BERT and ViT first / middle / last stages (reversible
and standard) from the installed copy of the reference (baseline/_ref, CPU only) and saves
their ``state_dict()`` - the content of the reference's ``latest_rank{r}.pth``
(BERT/src/ckpt_io.py:43-49).  Each must load into ``EncoderStage`` with no missing or
unexpected key after the wrapper aliases are folded, with every value unchanged.
"""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

GEN = r'''
import sys, torch
ref, model, out = sys.argv[1], sys.argv[2], sys.argv[3]
sys.path.insert(0, ref)
kw = dict(hidden_size=64, num_attention_heads=2, num_blocks=2, enable_amp=False, autocast_dtype=torch.float32,
          is_pareprop=False, num_classes=3, vocab_size=100, max_position_embeddings=16, type_vocab_size=2,
          img_size=32, patch_size=16, in_chans=3)
torch.manual_seed(0)
res = {}
if model == "bert":
    from models.bert_stages import BertFirstStage, BertMidStage, BertLastStage
    from models.normal_bert_stages import NormalBertFirstStage, NormalBertMidStage, NormalBertLastStage
    mods = {("reversible", 0): BertFirstStage, ("reversible", 1): BertMidStage, ("reversible", 2): BertLastStage,
            ("standard", 0): NormalBertFirstStage, ("standard", 1): NormalBertMidStage,
            ("standard", 2): NormalBertLastStage}
else:
    from models.vit_stages import ViTFirstStage, ViTMidStage, ViTLastStage
    from models.normal_vit_stages import NormalViTFirstStage, NormalViTMidStage, NormalViTLastStage
    mods = {("reversible", 0): ViTFirstStage, ("reversible", 1): ViTMidStage, ("reversible", 2): ViTLastStage,
            ("standard", 0): NormalViTFirstStage, ("standard", 1): NormalViTMidStage,
            ("standard", 2): NormalViTLastStage}
for key, cls in mods.items():
    res[key] = {k: v.clone() for k, v in cls(**kw).state_dict().items()}
torch.save(res, out)
'''


@pytest.mark.parametrize("model", ["bert", "vit"])
def test_reference_stage_state_dicts_load_strictly(tmp_path, model):
    sub = os.path.join(REF, "BERT" if model == "bert" else "Vit")
    if not os.path.isdir(sub):
        pytest.skip("the reference is not installed under baseline/_ref")
    out = tmp_path / "ref.pt"
    p = subprocess.run([sys.executable, "-c", GEN, sub, model, str(out)], capture_output=True, text=True,
                       timeout=300, cwd=str(tmp_path))
    assert p.returncode == 0, p.stderr[-3000:]
    ref = torch.load(out)

    from revpp.ckpt import strip_aliases
    from revpp.config import GlobalConfig
    from revpp.models.encoder import EncoderStage

    cfg = GlobalConfig(model=model, hidden_size=64, num_attention_heads=2, num_hidden_layers=6, num_classes=3,
                       vocab_size=100, max_position_embeddings=16, type_vocab_size=2, img_size=32, patch_size=16)
    for (kind, s), sd in ref.items():
        st = EncoderStage(cfg, s, 3, 2, kind)
        canon = strip_aliases(sd) if kind == "reversible" else sd
        missing, unexpected = st.load_state_dict(canon, strict=False)
        assert not missing and not unexpected, (kind, s, missing[:4], unexpected[:4])
        mine = st.state_dict()
        for k, v in canon.items():
            assert torch.equal(mine[k], v), (kind, s, k)
