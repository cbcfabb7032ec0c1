"""The C-ABI library loads and exports every entry point its header declares
(no GPU needed: nothing here launches a kernel)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "rembed_gpu.h"


def declared_symbols(header: Path) -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return set(re.findall(r"\b(rg_[a-z0-9_]+)\s*\(", text))


def test_header_declares_core_abi():
    syms = declared_symbols(HEADER)
    for s in ("rg_init", "rg_upload_weight", "rg_finalize", "rg_forward", "rg_free", "rg_free_string"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    from rembed_b200.embedder import library_path

    lib = ctypes.CDLL(str(library_path()))
    missing = [s for s in sorted(declared_symbols(HEADER)) if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from rembed_b200.embedder import SIGNATURES

    assert declared_symbols(HEADER) <= set(SIGNATURES), declared_symbols(HEADER) - set(SIGNATURES)


def test_error_strings_round_trip_without_gpu():
    """rg_init on a host without a usable device fails with a message, never aborts."""
    from rembed_b200 import synth
    from rembed_b200.embedder import Embedder, RembedError

    cfg = synth.preset("tiny-bert")
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is visible: covered by the GPU tests")
    except ImportError:
        pass
    with pytest.raises(RembedError):
        Embedder(cfg, {})


def test_python_mirror_takes_every_load_option():
    """The reference's Load options (rembed.go:67-121: WithInt8,
    WithInt8Activations, WithDiskWeights, WithDim, WithWorkers) are keyword
    arguments of load(); the Embedder exposes dim, model, quantized,
    quantized_activations, close and the context-manager protocol like the
    reference's Python binding."""
    import inspect

    from rembed_b200.embedder import Embedder, load

    params = inspect.signature(load).parameters
    for opt in ("int8", "int8_activations", "disk_weights", "dim", "workers"):
        assert opt in params, opt
    for attr in ("dim", "model", "quantized", "quantized_activations", "close", "__enter__", "__exit__",
                 "embed", "embed_tokens", "embed_packed", "submit"):
        assert hasattr(Embedder, attr), attr
