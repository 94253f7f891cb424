"""Host logic of ``bench.py`` (CPU only): argument forms the driver and the
sweeps use, bank composition and the attention pair count of the
extrapolated CPU baseline."""

import argparse
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def _args(*argv):
    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench.parse()
    finally:
        sys.argv = old


def test_defaults_are_one_gpu_p2p():
    a = _args()
    assert a.gpus == 1 and a.transport == ["p2p"] and a.workload == "prefill"


@pytest.mark.parametrize("text,want", [("p2p", ["p2p"]), ("nccl", ["nccl"]), ("p2p,nccl", ["p2p", "nccl"]),
                                       ("nccl, p2p", ["nccl", "p2p"])])
def test_transport_lists(text, want):
    assert bench._transports(text) == want
    assert _args("--transport", text).transport == want


@pytest.mark.parametrize("text", ["", "tcp", "p2p,p2p", "p2p,nccl,p2p"])
def test_transport_lists_rejected(text):
    with pytest.raises(argparse.ArgumentTypeError):
        bench._transports(text)


def test_request_tokens_uniform_and_mixed():
    assert bench.request_tokens(argparse.Namespace(prompt_tokens="32768", requests=4)) == [32768] * 4
    mixed = bench.request_tokens(argparse.Namespace(prompt_tokens="8192,32768,65536,131072", requests=4))
    assert mixed == [8192, 32768, 65536, 131072]
    with pytest.raises(SystemExit):
        bench.request_tokens(argparse.Namespace(prompt_tokens="0", requests=1))


def test_attention_pairs_of_a_chunk():
    # rows queries at positions h .. h+rows-1, each seeing keys 0 .. its position
    for h, rows in [(0, 1), (0, 2048), (30720, 2048), (7, 5)]:
        assert bench._pairs(h, rows) == sum(h + i + 1 for i in range(rows))
