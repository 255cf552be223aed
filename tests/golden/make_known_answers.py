"""Extract the reference's known-answer GEMM/GEMV/MatMul cases into a fixture.

Reads the reference's GTest sources AS TEXT (they need GTest/glog and a GPU,
neither of which is available for running them) and records each case's
input arrays, shapes and expected outputs:

  test/cuBlas/test_gemm/test_gemm.cpp     (GemmTest.ForwardFloatNoTranspose)
  test/cuBlas/test_gemv/test_gemv.cpp     (GemvTest.ForwardFloatNoTranspose)
  test/cuDNN/test_matmul/test_matmul.cpp  (MatMulTest.Forward2D, ForwardBatch3D)

Usage: python tests/golden/make_known_answers.py [REF_ROOT]
Writes tests/golden/known_answers.json next to this script.
"""
import json
import re
import sys
from pathlib import Path

REF = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
OUT = Path(__file__).resolve().parent / "known_answers.json"


def arrays(src: str, test_name: str) -> dict:
    """float NAME[n] = {...}; literals inside the body of TEST_F(..., test_name)."""
    start = src.index(test_name)
    nxt = src.find("TEST_F(", start + 1)
    body = src[start: nxt if nxt > 0 else len(src)]
    body = re.sub(r"//[^\n]*", "", body)
    out = {}
    for m in re.finditer(r"float\s+(\w+)\s*\[\s*\d+\s*\]\s*=\s*\{([^}]*)\}", body, re.S):
        vals = [float(v) for v in m.group(2).replace("\n", " ").split(",") if v.strip()]
        out[m.group(1)] = vals
    return out


def main() -> None:
    gemm = arrays((REF / "test/cuBlas/test_gemm/test_gemm.cpp").read_text(), "ForwardFloatNoTranspose")
    gemv = arrays((REF / "test/cuBlas/test_gemv/test_gemv.cpp").read_text(), "ForwardFloatNoTranspose")
    mm = (REF / "test/cuDNN/test_matmul/test_matmul.cpp").read_text()
    mm2 = arrays(mm, "Forward2D")
    mm3 = arrays(mm, "ForwardBatch3D")
    fixture = {
        "source": "reference GTest sources (known-answer cases), extracted as text",
        "gemm_2x3x4": {"file": "test/cuBlas/test_gemm/test_gemm.cpp", "M": 2, "K": 3, "N": 4,
                       "alpha": 1.0, "beta": 0.0, "A": gemm["h_input"], "B": gemm["h_weight"],
                       "expected": gemm["expected"], "tol": 1e-5},
        "gemv_2x3": {"file": "test/cuBlas/test_gemv/test_gemv.cpp", "M": 2, "N": 3, "alpha": 1.0, "beta": 0.0,
                     "A": gemv["h_input"], "x": gemv["h_weight"], "expected": gemv["expected"], "tol": 1e-5},
        "matmul_2d": {"file": "test/cuDNN/test_matmul/test_matmul.cpp", "M": 2, "K": 3, "N": 4,
                      "A": mm2["h_A"], "B": mm2["h_B"], "expected": mm2["expected"], "tol": 1e-5},
        "matmul_batch3d": {"file": "test/cuDNN/test_matmul/test_matmul.cpp", "batch": 2, "M": 2, "K": 3, "N": 4,
                           "A": mm3["h_A"], "B": mm3["h_B"], "expected": mm3["expected0"] + mm3["expected1"],
                           "tol": 1e-5},
    }
    OUT.write_text(json.dumps(fixture, indent=1) + "\n")
    print(OUT)


if __name__ == "__main__":
    main()
