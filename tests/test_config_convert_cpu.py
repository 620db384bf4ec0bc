"""The layout converter: a legacy single-section YAML becomes the sectioned
layout with comments kept next to their keys, a retired key dropped, a
misplaced key moved home, other sections copied as they are; the result loads
to the same settings; the shipped templates are fixed points."""
import glob
import os

import pytest
import yaml

from deltaserve_vllm_b200.config_convert import convert, main
from deltaserve_vllm_b200.config_loader import FINETUNE_SECTIONS

LEGACY = """# Serving config for a test

model:
  model: llama3-tiny   # tiny preset
  max_model_len: 512

# The finetune settings, all in one section
finetune:
  enable_finetuning: true
  # where the corpus lives
  data_path: data/train.txt
  learning_rate: 0.0002
  ttft_slo: 0.4        # seconds
  backward_sleep_seconds: 3
  ft_target_modules:
    - q_proj
    # value projection too
    - v_proj
  metrics_dir: logs/m

slo:
  max_tbt_slo: 0.08
  print_step_mode: true

engine:
  max_num_batched_tokens: 1024
"""


def test_legacy_layout_is_sectioned_with_comments_kept():
    new, notes = convert(LEGACY)
    raw = yaml.safe_load(new)
    assert "finetune" not in raw
    assert raw["finetune_param"] == {"enable_finetuning": True, "data_path": "data/train.txt",
                                     "learning_rate": 0.0002, "ft_target_modules": ["q_proj", "v_proj"]}
    assert raw["slo"] == {"ttft_slo": 0.4, "max_tbt_slo": 0.08}
    assert raw["debug"] == {"print_step_mode": True}          # moved out of slo
    assert raw["telemetry"] == {"metrics_dir": "logs/m"}
    assert raw["model"] == {"model": "llama3-tiny", "max_model_len": 512}
    assert raw["engine"] == {"max_num_batched_tokens": 1024}
    assert "backward_sleep_seconds" not in new
    assert any(n.startswith("dropped finetune.backward_sleep_seconds") for n in notes)
    assert "moved slo.print_step_mode -> debug.print_step_mode" in notes
    lines = new.splitlines()
    # comments stay directly above their keys, inline comments on their lines
    assert lines[lines.index("  data_path: data/train.txt") - 1] == "  # where the corpus lives"
    assert "  ttft_slo: 0.4        # seconds" in lines
    assert lines[lines.index("    - v_proj") - 1] == "    # value projection too"
    assert lines[lines.index("finetune_param:") - 1] == "# The finetune settings, all in one section"
    assert "  model: llama3-tiny   # tiny preset" in lines
    # finetune sections in their canonical order, where the first one stood
    order = [l[:-1] for l in lines if l.endswith(":") and not l.startswith(" ")]
    assert order == ["model", "finetune_param", "slo", "debug", "telemetry", "engine"]
    assert [s for s in order if s in FINETUNE_SECTIONS] == [s for s in FINETUNE_SECTIONS if s in order]


def test_shipped_templates_are_fixed_points():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    paths = sorted(glob.glob(os.path.join(root, "configs", "*.yaml")))
    assert paths
    for p in paths:
        text = open(p).read()
        assert convert(text)[0] == text, p


def test_unknown_finetune_key_is_refused(tmp_path):
    bad = tmp_path / "bad.yaml"
    bad.write_text("finetune:\n  not_a_setting: 1\n")
    with pytest.raises(ValueError, match="not a finetune setting"):
        main([str(bad), "--in-place"])
    assert bad.read_text() == "finetune:\n  not_a_setting: 1\n"


def test_in_place(tmp_path):
    p = tmp_path / "c.yaml"
    p.write_text(LEGACY)
    main([str(p), "--in-place"])
    assert "finetune_param:" in p.read_text()
    assert convert(p.read_text())[0] == p.read_text()
