"""The oracle's pins to the reference, re-run in the GPU suite.

The same checks as test_oracle.py (the C restatement against the golden
vectors the reference produced, and against the reference's own compiled
headers on random inputs), collected again under the gpu marker so that a
GPU run (`pytest -m gpu`) records, beside GPU == oracle, that the oracle ==
reference on the same machine.  They need no device."""
import pytest

import test_oracle as _pins

pytestmark = pytest.mark.gpu

test_attn_gqa_cache_bit_exact = _pins.test_attn_gqa_cache_bit_exact
test_empty_window_gives_zeros = _pins.test_empty_window_gives_zeros
test_bench_head_check = _pins.test_bench_head_check
test_vexp_bench_inputs = _pins.test_vexp_bench_inputs
test_norm_and_rope_close = _pins.test_norm_and_rope_close
test_layer_step_close = _pins.test_layer_step_close
test_layer_step_cache_full = _pins.test_layer_step_cache_full
test_reference_shim_matches_golden = _pins.test_reference_shim_matches_golden
test_port_equals_reference_random = _pins.test_port_equals_reference_random
test_prefill_oracle_matches_reference_golden = _pins.test_prefill_oracle_matches_reference_golden
test_q4_oracle_matches_reference_golden = _pins.test_q4_oracle_matches_reference_golden
test_q8_block_quantizer_matches_reference_golden = \
    _pins.test_q8_block_quantizer_matches_reference_golden
test_q8_block_quantizer_equals_reference_random = \
    _pins.test_q8_block_quantizer_equals_reference_random
