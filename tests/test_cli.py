"""The ``qwen-infra prefill`` surface without a GPU: argument validation
(``ValueError`` as the reference's ``config.py:63-73`` / ``cli.py:95-98``),
the ``--dry-run`` engine options (``cli.py:99-111``) and the output record
list (``cli.py:148-160``)."""

import json

import pytest
import torch

from qwen_infra_b200 import cli


def _dry(capsys, *extra):
    assert cli.main(["prefill", "--model", "tiny", "--dry-run", *extra]) == 0
    return json.loads(capsys.readouterr().out)


def test_dry_run_prints_the_engine_options(capsys):
    out = _dry(capsys, "--requests", "4", "--prompt-tokens", "2048", "--chunk-size", "512")
    eng = out["engine"]
    assert eng["model"] == "tiny" and eng["kv_cache_dtype"] == "nvfp4" and eng["max_num_batched_tokens"] == 512
    assert eng["profile"] == "vpp"
    extra = eng["additional_config"]
    assert extra["qwen_infra_vpp_transport"] == "p2p_copy_engine"
    assert extra["qwen_infra_vpp_resource_layout"] == "rank"
    assert extra["qwen_infra_vpp_slots"] == dict(source=2, destination=3, ring=7)
    assert out["requests"] == 4 and out["prompt_tokens"] == 2048


def test_nccl_transport_uses_edge_owned_slots(capsys):
    extra = _dry(capsys, "--transport", "nccl", "--resource-layout", "rank")["engine"]["additional_config"]
    assert extra["qwen_infra_vpp_transport"] == "nccl"
    assert extra["qwen_infra_vpp_resource_layout"] == "edge"  # rank-shared slots need the DMA transport
    extra = _dry(capsys, "--resource-layout", "edge")["engine"]["additional_config"]
    assert extra["qwen_infra_vpp_resource_layout"] == "edge"


def test_conventional_profile_has_no_fold_options(capsys):
    eng = _dry(capsys, "--profile", "cpp")["engine"]
    assert eng["profile"] == "cpp" and "additional_config" not in eng


@pytest.mark.parametrize("kwargs", [dict(profile="pp"), dict(model=""), dict(chunk_size=0), dict(chunk_size=16385),
                                    dict(max_model_len=1), dict(max_num_seqs=0), dict(gpu_memory_utilization=1.0),
                                    dict(gpu_memory_utilization=0.0), dict(transport="tcp"),
                                    dict(resource_layout="ring")])
def test_invalid_engine_options_raise_value_error(kwargs):
    base = dict(model="tiny")
    base.update(kwargs)
    with pytest.raises(ValueError):
        cli.PrefillConfig(**base).engine_options()


@pytest.mark.parametrize("argv", [["--requests", "0"], ["--prompt-tokens", "0"],
                                  ["--prompt-tokens", "32768", "--max-model-len", "32768"]])
def test_invalid_bank_arguments_raise_value_error(argv):
    with pytest.raises(ValueError):
        cli.main(["prefill", "--model", "tiny", "--dry-run", *argv])


def test_output_records_carry_the_reference_fields():
    outputs = [torch.ones(8, dtype=torch.bfloat16), torch.zeros(8, dtype=torch.bfloat16)]
    recs = cli._records(outputs, 2, [17, 3])
    assert [r["request_id"] for r in recs] == ["0", "1"]
    assert [r["token_ids"] for r in recs] == [[17], [3]]
    assert all(r["finished"] is True and r["text"] == "" for r in recs)
    assert recs[0]["final_hidden_norm"] == pytest.approx(8 ** 0.5) and recs[1]["final_hidden_norm"] == 0.0
    assert recs[0]["final_hidden_sha256"] != recs[1]["final_hidden_sha256"]
    json.dumps(recs)  # the printed list is plain JSON
