"""GPU: the language-model driver end to end on a small GPT-2 (2 layers), random init, synthetic
tokens: the run summary has the reference's keys in the reference's order (plus the driver's
"lsr" entry), and the training loss stays finite."""
import json
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "driver_golden.json").read_text())


def test_driver_runs_and_writes_the_reference_summary(tmp_path):
    from lsr import lm_driver
    out = tmp_path / "run.json"
    rc = lm_driver.main(["--muon-mode", "batched", "--init", "random", "--model-id", "gpt2",
                         "--config-overrides", "n_layer=2,n_embd=256,n_head=4", "--steps", "4",
                         "--warmup-steps", "1", "--seq-len", "128", "--grad-accum", "2",
                         "--train-token-cache", str(tmp_path / "absent.pt"), "--train-cache-tokens", "100000",
                         "--output", str(out)])
    assert rc == 0
    s = json.loads(out.read_text())
    assert list(s.keys()) == GOLD["summary_keys"] + ["lsr"]
    assert s["optimizer_structure"]["muon_matrix_count"] == 8
    assert s["median_muon_ms"] > 0 and s["median_step_ms"] >= s["median_optimizer_ms"]
    assert s["mean_measured_loss"] == s["mean_measured_loss"] and s["final_measured_loss"] < 20
    assert s["lsr"]["data"].startswith("synthetic")
