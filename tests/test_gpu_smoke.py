"""The round-end smoke check (__graft_entry__.smoke: one causal GQA bf16 forward + backward on cuda:0
against the CPU oracle) run as a GPU test, so that the suite catches a broken smoke path."""

import pytest

pytestmark = pytest.mark.gpu


def test_smoke_forward_backward_matches_oracle():
    import __graft_entry__

    __graft_entry__.smoke()
