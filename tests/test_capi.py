"""The C ABI library loads on a machine without a GPU, exports every function include/evie_cuda.h declares, and
rejects invalid arguments with a status and a message (no compute call needs a GPU here)."""
import ctypes as C
import os

import pytest

import evie_b200
from evie_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(evie_b200.LIB_PATH):
        evie_b200.build()
    return evie_b200.lib()


def test_exports_every_header_function(L):
    names = capi.header_functions(os.path.join(ROOT, "include", "evie_cuda.h"))
    assert len(names) >= 14
    missing = [n for n in names if getattr(L, n, None) is None]
    assert not missing, missing
    assert set(names) <= set(capi.SIGNATURES), "capi.SIGNATURES is missing a header function"


def test_argument_errors_have_messages(L):
    rc = L.evie_gdn_decode_step(None, None, None, None, None, None, None, 1, 1, 64, 128, None)
    assert rc == 1
    assert b"dk = dv = 128" in L.evie_last_global_error()
    rc = L.evie_gqa_decode_paged(None, None, None, None, None, None, None, 1, 16, 4, 128, 256, 4, 1.0, None)
    assert rc == 1 and b"head_dim 256" in L.evie_last_global_error()
    rc = L.evie_gdn_chunk_prefill(None, None, None, None, None, None, None, 1, 64, 1, 128, 128, 32, None)
    assert rc == 1 and b"chunk must be 64" in L.evie_last_global_error()
