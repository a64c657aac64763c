"""Regenerates the golden fixtures in this folder from go-tensor's own test data
(numbers and data files only, no code).

go-tensor's weight-loading test (weights/weights_test.go:18-74) checks its
forward pass of a small CNN against PyTorch's output for the same input. The
inputs, weights and expected outputs it uses live in
``weights/testdata/cnn_io.json`` and ``weights/testdata/cnn.safetensors``,
written by ``weights/testdata/gen_fixtures.py``. This script copies those
numbers (no code) into ``cnn_forward.json`` so the tests can run where the
reference tree is absent.

The CNN is Conv2d(1,2,3,pad 1) -> ReLU -> MaxPool2d(2) -> Flatten ->
Linear(32,3) on an input of shape [2,1,8,8]; parameter names follow the
reference's Sequential naming (0.weight, 0.bias, 4.weight, 4.bias).

Usage: python tests/golden/make_golden.py <go-tensor checkout>
"""
import json
import os
import shutil
import sys

from safetensors.numpy import load_file


def main(root: str) -> None:
    data = os.path.join(root, "weights", "testdata")
    with open(os.path.join(data, "cnn_io.json")) as f:
        io_vals = json.load(f)
    weights = load_file(os.path.join(data, "cnn.safetensors"))
    out = {
        "source": "go-tensor weights/testdata/cnn_io.json + cnn.safetensors (PyTorch float32 forward)",
        "tolerance": 1e-5,
        "input": io_vals["input"],
        "output": io_vals["output"],
        "params": {k: {"shape": list(v.shape), "values": [float(x) for x in v.reshape(-1)]}
                   for k, v in sorted(weights.items())},
    }
    here = os.path.dirname(os.path.abspath(__file__))
    dst = os.path.join(here, "cnn_forward.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", dst)

    # The safetensors decoder's known answers (weights/safetensors/
    # safetensors_test.go:12-21): zoo.safetensors holds one tensor of every
    # dtype the format defines, with metadata; zoo_expected.json its values.
    # cnn.safetensors is the PyTorch-written weight file of the CNN above.
    for name in ("zoo.safetensors", "cnn.safetensors"):
        shutil.copyfile(os.path.join(data, name), os.path.join(here, name))
        print("copied", name)
    with open(os.path.join(data, "zoo_expected.json")) as f:
        zoo = json.load(f)["safetensors"]
    with open(os.path.join(here, "zoo_safetensors_expected.json"), "w") as f:
        json.dump({"source": "go-tensor weights/testdata/zoo_expected.json, entry \"safetensors\"",
                   "metadata": {"note": "zoo", "format": "pt"}, "tensors": zoo}, f, indent=1)
    print("wrote zoo_safetensors_expected.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <go-tensor checkout>")
    main(sys.argv[1])
