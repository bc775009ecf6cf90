"""bench.py --impl reference runs the reference's CPU pipeline (the oracle's
restatement) and must never load the product's CUDA library: the driver's
reference-vs-product ratio is only meaningful if that arm maps no product
code.  CPU only; one short utterance through the whole audio pipeline."""
import json
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]

PROBE = r"""
import sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--utterances", "3",
            "--ref-utterances", "1"]
sys.path.insert(0, ROOT)
import bench
bench.main()
maps = open("/proc/self/maps").read()
print("MAPPED", int("libbark3_b200.so" in maps), int("libbark3_oracle.so" in maps))
"""


def test_reference_arm_maps_only_the_oracle():
    out = subprocess.run([sys.executable, "-c", PROBE.replace("ROOT", repr(str(ROOT)))], cwd=ROOT,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    line = json.loads(next(l for l in lines if l.startswith("{")))
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["config"]["utterances"] == 3 and line["scaling"] == "strong"
    assert line["cpu_baseline"]["kind"] == "port"
    mapped = next(l for l in lines if l.startswith("MAPPED")).split()
    assert mapped[1] == "0", "the reference arm loaded the product library"
    assert mapped[2] == "1"
