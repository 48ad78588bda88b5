"""Builds the committed golden fixtures from the reference checkout.

Run once where the reference checkout is available, giving its root:

    python tests/golden/make_fixtures.py <reference checkout>

It copies, unchanged, the reference's onnxruntime golden fixtures
(tests/testdata/{small,pad,mid}_{src.png,shadow.f32,output.f32},
manifest.json) and its two ONNX models (MIT-licensed GCDRNet weights,
src/Sdcb.SimdGcdrNet.Models/LICENSE) into tests/golden/, so that the tests,
smoke() and bench.py never read the reference tree at run time.
"""
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref: str) -> None:
    td = os.path.join(ref, "tests", "testdata")
    for tag in ("small", "pad", "mid"):
        for suffix in ("src.png", "shadow.f32", "output.f32"):
            shutil.copyfile(os.path.join(td, f"{tag}_{suffix}"), os.path.join(HERE, f"{tag}_{suffix}"))
    shutil.copyfile(os.path.join(td, "manifest.json"), os.path.join(HERE, "manifest.json"))
    os.makedirs(os.path.join(HERE, "models"), exist_ok=True)
    for m in ("gcdrnet_gcnet_sim.onnx", "gcdrnet_drnet_sim.onnx"):
        shutil.copyfile(os.path.join(td, "models", m), os.path.join(HERE, "models", m))
    shutil.copyfile(os.path.join(ref, "src", "Sdcb.SimdGcdrNet.Models", "LICENSE"),
                    os.path.join(HERE, "models", "LICENSE"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_fixtures.py <reference checkout root>")
    main(sys.argv[1])
