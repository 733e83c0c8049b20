"""Matrix Market input and the binary CSR cache, on the CPU.

spmvb_read_matrix_market must give the CSR the reference's own
read_matrix_market gives (run from oracle/_ref) bit for bit, and the same
error text, on files written here: every banner combination the reference
accepts, comments and blank lines, CRLF line ends, repeated entries (kept,
in the reference's order), symmetric mirrors, extra lines past the declared
count, number forms, and every error it reports."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
import spmvbench_b200 as S

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def write(tmp_path, name, text):
    p = tmp_path / name
    p.write_bytes(text.encode())
    return str(p)


def same_as_reference(path, threads=0):
    m, n, rp, ci, va = oracle.ref_read_matrix_market(path)
    A = S.read_matrix_market(path, threads=threads)
    assert (A.m, A.n) == (m, n)
    np.testing.assert_array_equal(A.rowptr, rp)
    np.testing.assert_array_equal(A.colind, ci)
    assert A.values.tobytes() == va.tobytes()
    return A


def random_mtx(rng, rows, cols, entries, field="real", symmetry="general", dup_frac=0.1, comments=True,
               crlf=False, fmt="{:.17g}"):
    lines = [f"%%MatrixMarket matrix coordinate {field} {symmetry}"]
    if comments:
        lines += ["% written by the test", "%"]
    lines.append(f"{rows} {cols} {entries}")
    ii = rng.integers(1, rows + 1, entries)
    jj = rng.integers(1, cols + 1, entries)
    if symmetry == "symmetric":
        ii, jj = np.maximum(ii, jj), np.minimum(ii, jj)
    ndup = int(entries * dup_frac)
    if ndup:
        k = rng.integers(0, entries, ndup)
        ii[-ndup:], jj[-ndup:] = ii[k], jj[k]
    vals = rng.standard_normal(entries) * 10.0 ** rng.integers(-5, 5, entries)
    for a, b, v in zip(ii, jj, vals):
        if field == "pattern":
            lines.append(f"{a} {b}")
        elif field == "integer":
            lines.append(f"{a} {b} {int(v * 1000)}")
        else:
            lines.append(f"{a} {b} {fmt.format(v)}")
        if comments and rng.random() < 0.01:
            lines.append("% interleaved comment")
        if comments and rng.random() < 0.01:
            lines.append("")
    end = "\r\n" if crlf else "\n"
    return end.join(lines) + end


@pytest.mark.parametrize("field", ["real", "integer", "pattern"])
@pytest.mark.parametrize("symmetry", ["general", "symmetric"])
def test_matches_reference(tmp_path, field, symmetry):
    rng = np.random.default_rng(hash((field, symmetry)) % 2**32)
    p = write(tmp_path, "a.mtx", random_mtx(rng, 300, 300 if symmetry == "symmetric" else 250, 4000,
                                            field, symmetry))
    same_as_reference(p)


def test_banner_case_crlf_and_number_forms(tmp_path):
    text = ("%%matrixmarket MATRIX Coordinate REAL General\r\n%\r\n4 5 8\r\n"
            "1 1 1\r\n1 2 -2.\r\n2 3 .5\r\n2 3 +7e2\r\n3 5 -1.25E-3\r\n4 4 3\r\n  4 1   0.1  \r\n"
            "1 1 123456789012345678901234567890\r\n")
    same_as_reference(write(tmp_path, "b.mtx", text))


def test_repeated_entries_keep_the_reference_order(tmp_path):
    # Rows long enough that std::sort does not fall back to insertion sort,
    # with many repeated columns.
    rng = np.random.default_rng(5)
    lines = ["%%MatrixMarket matrix coordinate real general", "3 40 3000"]
    for _ in range(3000):
        lines.append(f"{rng.integers(1, 4)} {rng.integers(1, 41)} {rng.standard_normal():.17g}")
    same_as_reference(write(tmp_path, "d.mtx", "\n".join(lines) + "\n"))


def test_lines_past_the_declared_count_are_ignored(tmp_path):
    text = ("%%MatrixMarket matrix coordinate real general\n3 3 2\n1 1 1\n2 2 2\n"
            "3 3 3\nnot an entry\n9 9 9\n")
    A = same_as_reference(write(tmp_path, "e.mtx", text))
    assert A.nnz == 2


def test_empty_matrices(tmp_path):
    same_as_reference(write(tmp_path, "z1.mtx", "%%MatrixMarket matrix coordinate real general\n0 0 0\n"))
    same_as_reference(write(tmp_path, "z2.mtx", "%%MatrixMarket matrix coordinate real general\n5 4 0\n"))


def test_many_threads_give_the_same_csr(tmp_path):
    rng = np.random.default_rng(9)
    # Several MiB, so the entry lines are split over several threads, with
    # symmetric mirrors and junk past the declared count at the end.
    text = random_mtx(rng, 20000, 20000, 250000, "real", "symmetric", dup_frac=0.05)
    text += "1 1 1\ngarbage line\n"
    p = write(tmp_path, "big.mtx", text)
    assert os.path.getsize(p) > 6 * 2**20
    ref = same_as_reference(p, threads=1)
    for t in (2, 3, 8, 0):
        A = S.read_matrix_market(p, threads=t)
        np.testing.assert_array_equal(A.rowptr, ref.rowptr)
        np.testing.assert_array_equal(A.colind, ref.colind)
        assert A.values.tobytes() == ref.values.tobytes()


def test_an_error_past_the_declared_count_in_another_thread_is_ignored(tmp_path):
    rng = np.random.default_rng(10)
    body = random_mtx(rng, 1000, 1000, 200000, "real", "general", comments=False)
    p = write(tmp_path, "tail.mtx", body + "1 1\n" * 50000 + "x y z\n")
    for t in (1, 4, 16):
        assert S.read_matrix_market(p, threads=t).nnz == 200000


BAD = [
    ("", "empty file"),
    ("\n", "missing %%MatrixMarket banner"),
    ("%%MatrixMarket vector coordinate real general\n1 1 1\n1 1 1\n", "only 'matrix' objects are supported"),
    ("%%MatrixMarket matrix array real general\n1 1\n1\n", "only 'coordinate' format is supported"),
    ("%%MatrixMarket matrix coordinate complex general\n1 1 1\n1 1 1 0\n", "complex matrices are not supported"),
    ("%%MatrixMarket matrix coordinate double general\n1 1 1\n1 1 1\n", "unsupported field type"),
    ("%%MatrixMarket matrix coordinate real skew-symmetric\n1 1 1\n1 1 1\n", "skew-symmetric"),
    ("%%MatrixMarket matrix coordinate real hermitian\n1 1 1\n1 1 1\n", "unsupported symmetry"),
    ("%%MatrixMarket matrix coordinate real\n1 1 1\n1 1 1\n", "unsupported symmetry"),
    ("%%MatrixMarket matrix coordinate real general\n% only comments\n", "missing size line"),
    ("%%MatrixMarket matrix coordinate real general\n3 x 3\n", "malformed size line"),
    ("%%MatrixMarket matrix coordinate real general\n-1 3 0\n", "negative dimensions"),
    ("%%MatrixMarket matrix coordinate real general\n3000000000 3 0\n", "dimensions exceed int32"),
    ("%%MatrixMarket matrix coordinate real general\n3 3 1\n1\n", "malformed entry line"),
    ("%%MatrixMarket matrix coordinate real general\n3 3 1\n1 2\n", "expected a value on entry line"),
    ("%%MatrixMarket matrix coordinate real general\n3 3 1\n1 2 nan\n", "expected a value on entry line"),
    ("%%MatrixMarket matrix coordinate real general\n3 3 1\n4 1 1\n", "index out of range"),
    ("%%MatrixMarket matrix coordinate real general\n3 3 1\n0 1 1\n", "index out of range"),
    ("%%MatrixMarket matrix coordinate real general\n3 3 1\n   \n", "malformed entry line"),
    ("%%MatrixMarket matrix coordinate real general\n3 3 3\n1 1 1\n2 2 2\n", "expected 3 entries but found 2"),
]


@pytest.mark.parametrize("text,what", BAD, ids=[w for _, w in BAD])
def test_errors_match_the_reference(tmp_path, text, what):
    p = write(tmp_path, "bad.mtx", text)
    with pytest.raises(RuntimeError) as ref_err:
        oracle.ref_read_matrix_market(p)
    with pytest.raises(S.SpmvbError) as err:
        S.read_matrix_market(p)
    assert err.value.status == 2
    assert what in str(ref_err.value)
    assert str(ref_err.value) in str(err.value)


def test_missing_file(tmp_path):
    p = str(tmp_path / "nope.mtx")
    with pytest.raises(RuntimeError) as ref_err:
        oracle.ref_read_matrix_market(p)
    with pytest.raises(S.SpmvbError) as err:
        S.read_matrix_market(p)
    assert err.value.status == 9 and str(ref_err.value) in str(err.value)


def test_csr_cache_round_trip(tmp_path):
    A = S.generate(3, seed=3, scale_rows=20000)
    p = str(tmp_path / "a.csrbin")
    S.write_csr_cache(p, A)
    assert os.path.getsize(p) == 40 + 4 * (A.m + 1) + 12 * A.nnz
    B = S.read_csr_cache(p)
    assert (B.m, B.n) == (A.m, A.n)
    np.testing.assert_array_equal(B.rowptr, A.rowptr)
    np.testing.assert_array_equal(B.colind, A.colind)
    assert B.values.tobytes() == A.values.tobytes()


def test_csr_cache_rejects_bad_files(tmp_path):
    A = S.generate(1, seed=3, scale_rows=1000)
    p = tmp_path / "a.csrbin"
    S.write_csr_cache(str(p), A)
    raw = bytearray(p.read_bytes())
    (tmp_path / "trunc.csrbin").write_bytes(bytes(raw[:-8]))
    bad_magic = bytes(b"X" + raw[1:])
    (tmp_path / "magic.csrbin").write_bytes(bad_magic)
    corrupt = bytearray(raw)
    corrupt[40 + 4 * (A.m + 1)] = 0xFF  # first colind out of range
    corrupt[40 + 4 * (A.m + 1) + 3] = 0x7F
    (tmp_path / "corrupt.csrbin").write_bytes(bytes(corrupt))
    for name in ("trunc", "magic", "corrupt"):
        with pytest.raises(S.SpmvbError) as e:
            S.read_csr_cache(str(tmp_path / f"{name}.csrbin"))
        assert e.value.status == 2
    with pytest.raises(S.SpmvbError) as e:
        S.read_csr_cache(str(tmp_path / "missing.csrbin"))
    assert e.value.status == 9


def test_csr_cache_header_cannot_claim_more_than_the_file(tmp_path):
    """A damaged header (nnz or m near 2^31) in a small file is refused from
    the file size before any allocation, not after zeroing tens of GB."""
    import struct
    import time
    A = S.generate(1, seed=4, scale_rows=200)
    p = tmp_path / "a.csrbin"
    S.write_csr_cache(str(p), A)
    raw = bytearray(p.read_bytes())
    for off, fmt, value in ((24, "<q", 2**31 - 1), (16, "<i", 2**31 - 2)):  # nnz, m
        bad = bytearray(raw)
        struct.pack_into(fmt, bad, off, value)
        q = tmp_path / f"big{off}.csrbin"
        q.write_bytes(bytes(bad))
        t0 = time.perf_counter()
        with pytest.raises(S.SpmvbError, match="truncated") as e:
            S.read_csr_cache(str(q))
        assert e.value.status == 2 and time.perf_counter() - t0 < 1.0


def test_csr_cache_random_damage(tmp_path):
    """Truncations and byte flips anywhere: every read either fails with an
    error status or returns a CSR that passes validation."""
    A = S.generate(1, seed=5, scale_rows=300)
    p = tmp_path / "a.csrbin"
    S.write_csr_cache(str(p), A)
    raw = p.read_bytes()
    rng = np.random.default_rng(6)
    q = tmp_path / "f.csrbin"
    for t in range(600):
        b = bytearray(raw)
        if t % 3 == 0:
            b = b[: int(rng.integers(0, len(b)))]
        else:
            lo = 0 if t % 3 == 1 else 40
            for _ in range(int(rng.integers(1, 5))):
                b[int(rng.integers(lo if lo < len(b) else 0, len(b)))] = int(rng.integers(0, 256))
        q.write_bytes(bytes(b))
        try:
            B = S.read_csr_cache(str(q))
        except S.SpmvbError:
            continue
        S.csr_validate(B)
    bad = S.CsrMatrix(2, 2, np.array([0, 2, 1], np.int32), np.array([0, 1], np.int32), np.ones(2))
    with pytest.raises(S.SpmvbError):
        S.write_csr_cache(str(tmp_path / "never.csrbin"), bad)


# Value texts around the edges of `istream >> double` (std::num_get): signs,
# bare points, exponents without digits, overflow and underflow, special
# names, hexadecimal, separators and trailing text.
VALUE_FORMS = ["1", "-0", "+3.5", ".5", "5.", "1E-3", "1E+05", "0.1e1", "000001", "-000.000", "-.5e+1",
               "inf", "-inf", "nan", "NaN", "Infinity", "0x1p3", "1,5", "1_0", "--1", "+.", ".", ".e5", "e5",
               "1.5e", "1.5E", "1.5e+", "1.5e-", "1.5e++5", "5e", "1.5e5.3", "1.5ex", "1.5x", "1.5 junk",
               "1e400", "-1e400", "1.8e308", "1.7976931348623158e308", "1e308", "9" * 400,
               "1e-400", "-1e-400", "4.9e-324", "2.5e-324", "2.4e-324", "1e0000000000000000001",
               "  7", "7  ", "\t7"]


@pytest.mark.parametrize("form", VALUE_FORMS)
def test_value_forms_match_reference(tmp_path, form):
    """Each value text either reads as the reference reads it, bit for bit, or
    fails with the reference's message."""
    p = write(tmp_path, "v.mtx", f"%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 {form}\n2 2 2.0\n")
    try:
        ref = oracle.ref_read_matrix_market(p)
        ref_err = None
    except RuntimeError as e:
        ref_err = str(e)
    if ref_err is None:
        A = S.read_matrix_market(p)
        assert A.values.tobytes() == ref[4].tobytes()
    else:
        with pytest.raises(S.SpmvbError) as ei:
            S.read_matrix_market(p)
        assert ref_err in str(ei.value)


def _same_outcome(path):
    """The reference's CSR bit for bit, or its error text within ours."""
    try:
        ref = oracle.ref_read_matrix_market(path)
    except RuntimeError as e:
        with pytest.raises(S.SpmvbError) as ei:
            S.read_matrix_market(path)
        assert str(e) in str(ei.value)
        return
    A = S.read_matrix_market(path)
    assert (A.m, A.n) == ref[:2]
    np.testing.assert_array_equal(A.rowptr, ref[2])
    np.testing.assert_array_equal(A.colind, ref[3])
    assert A.values.tobytes() == ref[4].tobytes()


INDEX_FORMS = ["1", "+1", "01", "1.0", "1e0", "-1", "0", "3", "9999999999999999999", "18446744073709551616",
               "1x", "x", "0x1", " 1"]


@pytest.mark.parametrize("form", INDEX_FORMS)
def test_index_forms_match_reference(tmp_path, form):
    _same_outcome(write(tmp_path, "r.mtx", f"%%MatrixMarket matrix coordinate real general\n2 2 2\n{form} 1 5.0\n"
                                           "2 2 2.0\n"))
    _same_outcome(write(tmp_path, "c.mtx", f"%%MatrixMarket matrix coordinate pattern general\n2 2 2\n1 {form}\n"
                                           "2 2\n"))


SIZE_LINES = ["2 2 2", "2 2", "2", "2 2 2 extra", "-2 2 2", "2 -2 2", "2 2 -2", "2.5 2 2", "2 2 2.5",
              "99999999999 2 2", "2 99999999999 2", "2147483647 1 0", "2147483648 1 0", "0 0 0", "2 2 3", "2 2 1",
              "+2 +2 +2", "2e0 2 2", "2 2 9999999999999999999999"]


@pytest.mark.parametrize("line", SIZE_LINES)
def test_size_lines_match_reference(tmp_path, line):
    _same_outcome(write(tmp_path, "s.mtx", f"%%MatrixMarket matrix coordinate real general\n{line}\n1 1 5.0\n"
                                           "2 2 2.0\n"))


BANNERS = ["%%MatrixMarket matrix coordinate real general", "%%matrixmarket MATRIX Coordinate REAL General",
           "%%MatrixMarket matrix coordinate real", "%%MatrixMarket matrix coordinate", "%%MatrixMarket matrix",
           "%%MatrixMarket", "%MatrixMarket matrix coordinate real general",
           "%%MatrixMarket vector coordinate real general", "%%MatrixMarket matrix array real general",
           "%%MatrixMarket matrix coordinate complex general", "%%MatrixMarket matrix coordinate real hermitian",
           "%%MatrixMarket matrix coordinate real skew-symmetric", "%%MatrixMarket matrix coordinate double general",
           "%%MatrixMarket matrix coordinate real general extra", "  %%MatrixMarket matrix coordinate real general",
           "%%MatrixMarket  matrix\tcoordinate real general"]


@pytest.mark.parametrize("banner", BANNERS)
def test_banners_match_reference(tmp_path, banner):
    _same_outcome(write(tmp_path, "b.mtx", f"{banner}\n2 2 2\n1 1 5.0\n2 2 2.0\n"))
