"""Build-time check of the attention kernel's register count (no GPU): the
setmaxnreg split of flash_attn_fwd_kernel assumes 168 registers per thread at
launch, and sion_b200.build refuses a compile that ptxas gave another count."""
import pytest

from sion_b200.build import FA_REGS_LAUNCH, check_attention_registers

_LOG = """ptxas info    : Compiling entry function '_ZN11felix_sm1004attn21flash_attn_fwd_kernelILi128ELi1EEEv' for 'sm_100a'
ptxas info    : Function properties for _ZN11felix_sm1004attn21flash_attn_fwd_kernelILi128ELi1EEEv
    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used {n} registers, used 1 barriers
ptxas info    : Compiling entry function '_ZN5other6kernelEv' for 'sm_100a'
ptxas info    : Used 40 registers, used 1 barriers
"""


def test_expected_register_count_passes():
    check_attention_registers(_LOG.format(n=FA_REGS_LAUNCH))


def test_other_register_count_is_refused():
    with pytest.raises(RuntimeError, match="setmaxnreg split assumes 168"):
        check_attention_registers(_LOG.format(n=152))
