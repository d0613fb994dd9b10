"""The bench's roofline numerators, pinned to the figures its JSON line and
the documentation quote: algorithmic bytes of a step of the non-GEMM
sequence, GEMM FLOPs of the encoder stack, multiply-adds of a fused decode
iteration. A change to any formula shows up here before it shifts a
reported fraction."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_step_bytes_of_the_headline_workload():
    # 256 utterances x 375 frames x 24 blocks: 536.27 GB per step
    assert bench.step_bytes(256 * 375, 375, 256, 24) == 536_271_716_352


def test_encoder_gemm_flops_per_frame():
    per_frame = bench.encoder_gemm_flops(375) / 375
    assert abs(per_frame - 55.5e6) < 0.1e6, per_frame


def test_decode_multiply_adds():
    assert bench.decode_fmas(1, 0) == 2 * 2 * 2560 * 640          # both LSTM layers' gate products
    assert bench.decode_fmas(0, 1) == 640 * 640 + 640 * 1025      # pred + out products
    assert bench.decode_fmas(256, 256) == 256 * (6_553_600 + 1_065_600)


def test_ragged_bytes_are_the_items_sum():
    # a uniform batch counted item by item equals the batch formula
    assert bench.ragged_step_bytes([375] * 256, 24) == bench.step_bytes(256 * 375, 375, 256, 24)
    # config 3: 8 chunks (408, 416 x 6, 408) x 24 blocks
    lens = bench.CONFIG3_LENGTHS
    assert sum(lens) == 3312 and len(lens) == 8
    assert bench.ragged_step_bytes(lens, 24) == sum(bench.step_bytes(T, T, 1, 24) for T in lens)
