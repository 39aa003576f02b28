"""Writes tests/golden/kat.json: the known-answer vectors of the reference's own
test files for the hot path, transcribed with their file:line.

The reference is pure Julia and no Julia toolchain exists on either machine,
so the vectors are read from the test sources as text (inputs and expected
outputs exactly as those tests state them) rather than produced by running
them.  Run `python tests/golden/make_golden.py` to regenerate.
"""
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))

# A = [1 0 2; 0 3 0; 4 0 5] in CSR, used across the reference's kernel tests.
A_ONE = {"m": 3, "n": 3, "rowptr": [1, 3, 4, 6], "colind": [1, 3, 2, 1, 3],
         "val": [1.0, 2.0, 3.0, 4.0, 5.0], "base": 1}
A_ZERO = {"m": 3, "n": 3, "rowptr": [0, 2, 3, 5], "colind": [0, 2, 1, 0, 2],
          "val": [1.0, 2.0, 3.0, 4.0, 5.0], "base": 0}

KATS = {
    "spmv_csr_onebased": {
        "source": "test/test_emitter.jl:85-102; test/test_emitter_cuda.jl:46-62; test/test_cuda.jl:272-282",
        "A": A_ONE, "x": [1.0, 2.0, 3.0], "alpha": 1.0, "beta": 0.0, "y": [7.0, 6.0, 19.0]},
    "spmv_csr_zerobased": {
        "source": "test/test_emitter.jl:106-123",
        "A": A_ZERO, "x": [1.0, 2.0, 3.0], "alpha": 1.0, "beta": 0.0, "y": [7.0, 6.0, 19.0]},
    "spmv_dcsr_onebased": {
        "source": "test/test_emitter.jl:127-157 (row 2 not stored, y starts at zero)",
        "m": 3, "n": 3, "row_ids": [1, 3], "fibptr": [1, 3, 5], "colind": [1, 3, 1, 3],
        "val": [1.0, 2.0, 4.0, 5.0], "base": 1, "x": [1.0, 2.0, 3.0], "y0": [0.0, 0.0, 0.0],
        "alpha": 1.0, "beta": 0.0, "y": [7.0, 0.0, 19.0]},
    "spmv_coo_onebased": {
        "source": "test/test_emitter.jl:161-192",
        "m": 3, "n": 3, "rows": [1, 1, 2, 3, 3], "cols": [1, 3, 2, 1, 3],
        "val": [1.0, 2.0, 3.0, 4.0, 5.0], "base": 1, "x": [1.0, 2.0, 3.0],
        "alpha": 1.0, "beta": 0.0, "y": [7.0, 6.0, 19.0]},
    "spmm_csr_onebased": {
        "source": "test/test_emitter.jl:196-228; test/test_cuda.jl:304-314",
        "A": A_ONE, "B": [[1.0, 0.0], [2.0, 1.0], [0.0, 3.0]], "alpha": 1.0, "beta": 0.0,
        "C": [[1.0, 6.0], [6.0, 3.0], [4.0, 15.0]]},
    "sddmm_csr_onebased": {
        "source": "test/test_emitter.jl:264-287; test/test_cuda.jl:417-432",
        "A": [[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]],
        "B": [[1.0, 0.0, 1.0], [0.0, 1.0, 1.0]],
        "C": {"m": 3, "n": 3, "rowptr": [1, 3, 4, 6], "colind": [1, 3, 2, 1, 3],
              "val": [1.0, 1.0, 1.0, 1.0, 1.0], "base": 1},
        "alpha": 1.0, "beta": 0.0, "out": [1.0, 1.0, 1.0, 1.0, 2.0]},
    "spgemm_csr": {
        "source": "test/test_cuda.jl:436-451 (C = A*A, Float32)",
        "A": A_ONE, "C_dense": [[9.0, 0.0, 12.0], [0.0, 9.0, 0.0], [24.0, 0.0, 33.0]]},
    "convert_fixture_3x4": {
        "source": "test/test_convert.jl:3-9 (fixture), :44-58 (CSR->CSC buffers)",
        "A": {"m": 3, "n": 4, "rowptr": [0, 2, 3, 5], "colind": [0, 2, 1, 0, 2],
              "val": [1.0, 2.0, 3.0, 4.0, 5.0], "base": 0},
        "csc": {"colptr": [0, 2, 3, 5, 5], "rowind": [0, 2, 1, 0, 2],
                "val": [1.0, 4.0, 3.0, 2.0, 5.0]},
        "decomposer_visits": [[[0, 0], 1.0], [[0, 2], 2.0], [[1, 1], 3.0], [[2, 0], 4.0],
                              [[2, 2], 5.0]]},
    "bsm_diagonal": {
        "source": "test/test_emitter_cuda.jl:297-310 (BlockSparseMatrix([A1 nothing; nothing A2]))",
        "blocks": {"0,0": {"m": 2, "n": 3, "rowptr": [1, 3, 4], "colind": [1, 3, 2],
                           "val": [1.0, 2.0, 3.0], "base": 1},
                   "1,1": {"m": 2, "n": 3, "rowptr": [1, 2, 4], "colind": [2, 1, 3],
                           "val": [1.0, 1.0, 1.0], "base": 1}},
        "grid": [2, 2], "x": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], "y": [7.0, 6.0, 5.0, 10.0]},
    "bsm_accumulate": {
        "source": "test/test_emitter_cuda.jl:312-322 (BlockSparseMatrix([A1 A2]))",
        "blocks": {"0,0": {"m": 2, "n": 3, "rowptr": [1, 3, 4], "colind": [1, 3, 2],
                           "val": [1.0, 2.0, 3.0], "base": 1},
                   "0,1": {"m": 2, "n": 3, "rowptr": [1, 2, 4], "colind": [2, 1, 3],
                           "val": [1.0, 1.0, 1.0], "base": 1}},
        "grid": [1, 2], "x": [1.0, 2.0, 3.0, 1.0, 2.0, 3.0], "y": [9.0, 10.0]},
    "bsr_level_maps": {
        "source": "test/test_formats.jl:59-60,70,87-88,167-172",
        "dim2lvl": [
            {"format": "BSRRight", "block": [2, 2], "dims": [2, 1], "lvl": [1, 0, 0, 1]},
            {"format": "BSRLeft", "block": [2, 2], "dims": [2, 1], "lvl": [1, 0, 1, 0]},
            {"format": "CSR", "dims": [2, 1], "lvl": [2, 1]},
            {"format": "CSC", "dims": [2, 1], "lvl": [1, 2]}],
        "dim2lvl_as_size": [
            {"format": "BSRRight", "block": [2, 2], "dims": [8, 4], "lvl": [4, 2, 2, 2]},
            {"format": "CSR", "dims": [8, 4], "lvl": [8, 4]},
            {"format": "CSC", "dims": [8, 4], "lvl": [4, 8]}],
        "lvl2dim": [
            {"format": "BSRRight", "block": [2, 2], "lvl": [1, 0, 0, 1], "dims": [2, 1]},
            {"format": "BSRLeft", "block": [2, 2], "lvl": [1, 0, 1, 0], "dims": [2, 1]},
            {"format": "CSC", "lvl": [1, 2], "dims": [2, 1]}]},
}


def main():
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(KATS, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main()
