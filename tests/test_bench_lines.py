"""The generate/bench output-line contract of the reference's `bench` command
(src/minicpmo/qwen3.uya:2374-2399 for the rate, duration and microsecond
lines, 2950-2971 for their order): format_bench_lines against lines built here
from the reference's printf formats and its integer arithmetic."""
from __future__ import annotations

import re

import pytest


def _ref_rate(label, units, micros, reps):
    # qwen3_bench_rate_x1000 / qwen3_bench_print_rate: u64 arithmetic
    scaled = 0 if micros == 0 else units * 1_000_000_000 // micros
    return (f"bench {label}: {scaled // 1000}.{scaled % 1000:03d} tokens/s units={units} "
            f"ms={micros // 1000}.{micros % 1000:03d} repetitions={reps}")


STATS = dict(backend_init_us=1234567, host_to_device_bytes=11, device_to_host_bytes=22, weight_upload_bytes=33,
             uploaded_weight_count=7, kv_device_bytes=44)


@pytest.mark.parametrize("prompt_us,decode_us,first_us,reps", [
    (123456.7, 987654.3, 1500.9, 1),    # fractional microseconds truncate first, as the reference's u64 do
    (999.999, 1000.0, 0.0, 3),
    (0.0, 1.0, 2.0, 2),                 # zero time: rate 0, as qwen3_bench_rate_x1000
    (3_000_000_123.0, 7.0, 10.0, 5),
])
def test_bench_lines_match_reference_formats(pkg, prompt_us, decode_us, first_us, reps):
    from minicpmo_b200.qwen3 import format_bench_lines

    r = {"prompt_tokens": 64 * reps, "prompt_us": prompt_us, "decode_tokens": 128 * reps, "decode_us": decode_us,
         "first_token_us": first_us}
    lines = format_bench_lines(r, reps, STATS)
    assert lines[0] == _ref_rate("text_prompt", 64 * reps, int(prompt_us), reps)
    assert lines[1] == _ref_rate("text_decode", 128 * reps, int(decode_us), reps)
    fu = int(first_us)
    assert lines[2] == f"bench first_token: us={fu} avg_us={fu // reps} repetitions={reps}"
    assert lines[3].startswith("bench backend: ") and "weights_uploaded=7" in lines[3]
    assert lines[4] == ("bench transfer: backend_init_ms=1234.567 host_to_device_bytes=11 device_to_host_bytes=22 "
                        "weights_device_bytes=33 kv_device_bytes=44")
    assert lines[-1] == "bench: PASS"


def test_bench_rate_integer_division_differs_from_float(pkg):
    """A case where dividing by the float time would round the other way: the line follows the
    reference's integer microseconds."""
    from minicpmo_b200.qwen3 import format_bench_lines

    r = {"prompt_tokens": 3, "prompt_us": 7.9, "decode_tokens": 1, "decode_us": 1.0, "first_token_us": 1.0}
    line = format_bench_lines(r, 1, STATS)[0]
    assert line.startswith("bench text_prompt: 428571.428 tokens/s units=3 ms=0.007 ")  # 7.9 us as a float: 379746.835
    assert re.fullmatch(r"bench text_prompt: \d+\.\d{3} tokens/s units=\d+ ms=\d+\.\d{3} repetitions=\d+", line)
