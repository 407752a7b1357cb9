"""bench.py's own arithmetic and rules, on the CPU.

The workload constants the bench divides by (weight bytes per step, KV bytes per position, the
handoff and prefill units) follow from the model shape BASELINE names; config 4's past lengths
leave room for its 128 greedy steps inside the S=512 cache; the warm-up rule is enforced; the
clock record that decides whether a run is kept is parsed as nvidia-smi writes it; and the
host-staged handoff baseline reports what its JSON line claims.
"""
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "rngd-pd_b200")]

import bench  # noqa: E402
from rngd_pd.engines.model import ModelConfig  # noqa: E402


def test_workload_units_follow_the_model_shape():
    c = ModelConfig.llama31_8b()
    H, M, NH, NKV, HD, L, V = c.hidden, c.inter, c.n_heads, c.n_kv, c.head_dim, c.n_layers, c.vocab
    layer = (H * NH * HD + 2 * H * NKV * HD + NH * HD * H + 3 * H * M) * 2   # bf16 projections
    assert layer == 436_207_616
    assert bench.WEIGHT_BYTES == L * layer + V * H * 2                       # + lm_head
    assert bench.KV_BYTES_PER_POS == L * NKV * HD * 2 * 2                    # K and V, bf16
    assert bench.handoff_bytes(c) == 67_108_864                              # one 512-token request
    assert abs(bench.prefill_flops(c, 256) - 3.59e12) < 0.01e12              # config 2's pass


def test_config4_lengths_leave_room_for_128_steps():
    lens, toks = bench.lengths_and_tokens(cpu=True)
    assert len(lens) == len(toks) == bench.B
    assert all(64 <= n <= 384 for n in lens) and max(lens) + 128 <= bench.S
    assert all(0 <= t < 128256 for t in toks)
    assert (lens, toks) == bench.lengths_and_tokens(cpu=True)                 # seeded


def test_warmup_below_three_is_refused():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--warmup", "2"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode != 0 and "--warmup must be >= 3" in r.stderr


class _Done:
    def terminate(self):
        pass

    def wait(self):
        return 0


def test_clock_record_parser(tmp_path):
    """Median SM clock under load, the max clock, and which throttle reasons were ever active
    (a hardware or thermal slowdown rejects a run; the power cap is kept and noted)."""
    path = tmp_path / "clocks.csv"
    path.write_text("0, 1965, 1965, 701.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active\n"
                    "0, 1950, 1965, 990.2, 0x0000000000000004, Not Active, Not Active, Not Active, Active\n"
                    "0, 1935, 1965, 995.0, 0x0000000000000048, Not Active, Active, Not Active, Active\n"
                    "[N/A]\n")
    c = bench.Clocks.__new__(bench.Clocks)
    c.f, c.p = open(path), _Done()
    got = c.stop()
    assert got == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["hw_thermal_slowdown", "sw_power_cap"],
                   "samples": 3}
    assert not path.exists()                                                  # the record is removed


def test_host_staged_handoff_baseline_line():
    got = bench.handoff_cpu_baseline()
    assert got["unit"] == "GB/s" and got["kind"] == "port" and got["cores"] == 1 and got["value"] > 0
