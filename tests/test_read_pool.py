"""The reads-in-flight pool's scheduling rules (tierstream_b200/csrc/read_pool_check.cpp, through tsb_test_read_pool):
with a fake read that blocks until released, landing reads wait behind demand reads, the reserve keeps one reader free
of them, the cap counts the reads that run, cancel drops only a landing read that has not started, and a demand's end
of a queued landing read runs it before the other queued demand reads. No file and no device."""
import pytest

from tierstream_b200 import abi


@pytest.mark.parametrize("repeat", range(5))
def test_read_pool_rules(repeat):
    lib = abi.load()
    assert lib.tsb_test_read_pool() == abi.SS_OK, lib.ss_last_error().decode()
