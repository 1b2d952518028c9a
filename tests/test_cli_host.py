"""CPU: the native atlas_dynamic_infer's tokenizer (-1.7-atlas---apollo_b200/host/cli.c,
built here as a library with ATLAS_CLI_LIBRARY) gives the reference's
tokenize_prompt ids (src/brain_runtime.c:636-840, compiled in place) for the
same file, across the pre-tokenization cases: the chat template's special
tokens, runs of spaces / tabs / newlines, contractions, digit runs, punctuation
and bytes >= 128."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import atlas_cuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "-1.7-atlas---apollo_b200", "host", "cli.c")

TEXTS = [
    "<|im_start|>user\nHello there, how are you?<|im_end|>\n<|im_start|>assistant\n",
    "plain text without a template",
    "  two leading spaces and   three inside  ",
    "tabs\t\tand\nnew\r\nlines\n\n\nend",
    "Don't, I'm, we'll, they've, she'd, it's, you're, IT'S",
    "digits 1234567 and 12 3 4567890 x1y22z333",
    "punctuation!!! ??? ... ;;; (parens) [brackets] {braces} @#$%^&*",
    "unicode: café naïve 日本語 \U0001F600 ½",
    "<|im_start|>system\nYou are helpful.<|im_end|>\n<|im_start|>user\nq<|im_end|>\n<|im_start|>assistant\n",
    "<|notaspecial|> stays text",
    "trailing space ",
    "x",
]


@pytest.fixture(scope="module")
def cli_lib(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("cli") / "libclitok.so")
    subprocess.run(["gcc", "-O2", "-std=gnu11", "-shared", "-fPIC", "-DATLAS_CLI_LIBRARY",
                    "-I" + os.path.join(ROOT, "include"), CLI, "-o", out, "-lm"], check=True)
    L = ctypes.CDLL(out)
    L.cli_tokenize.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64]
    return L


def test_cli_tokenizer_matches_reference(cli_lib, ref, model_dir):
    path = os.path.join(str(model_dir), "cli_tok.gguf")
    if not os.path.exists(path):
        atlas_cuda.write_synthetic_gguf(path, hidden=512, layers=1, q_heads=4, kv_heads=2, ffn=768, vocab=8192,
                                        context_length=512, seed=31)
    ref.open(path)
    ref.L.ref_tokenize.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64]
    try:
        for text in TEXTS:
            b = text.encode()
            want = np.zeros(4096, np.uint32)
            got = np.zeros(4096, np.uint32)
            nw = ref.L.ref_tokenize(b, want.ctypes.data, 4096)
            ng = cli_lib.cli_tokenize(path.encode(), b, got.ctypes.data, 4096)
            assert ng == nw, (text, ng, nw)
            np.testing.assert_array_equal(got[:ng], want[:nw], err_msg=text)
    finally:
        ref.close()
