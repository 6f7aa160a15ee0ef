"""The header-only C++ layer (include/ckks_b200.hpp) compiles and links
against the C ABI library (CPU only: nothing is executed)."""

import os
import shutil
import subprocess

from private_genomic_dnagpt_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include "ckks_b200.hpp"
#include <cstdio>
int main() {
  using namespace ckks_b200;
  CCParams p;
  p.ring_dim_log = 12;
  p.multiplicative_depth = 5;
  auto cc = GenCryptoContext(p);
  cc->KeyGen();
  cc->EvalMultKeyGen();
  cc->EvalRotateKeyGen({1, 2, 3});  // AccumulateSum(4, 1) ladder: 1, 2, 3
  auto ct = cc->Encrypt(cc->MakeCKKSPackedPlaintext({1.0, 2.0, 3.0}));
  auto r = cc->EvalRotate(cc->EvalMult(ct, ct), 1);
  auto s = cc->AccumulateSum(cc->EvalAdd(r, 0.5), 4, 1);
  auto v = cc->Decrypt(cc->LevelReduce(s, 2))->GetRealPackedValue();
  std::printf("%zu %u %.9f\n", v.size(), s->GetLevel(), v[0]);
  return 0;
}
"""


def test_cpp_layer_compiles_and_links(tmp_path):
    lib = build()
    cxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++")
    src = tmp_path / "prog.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "prog"
    r = subprocess.run([cxx, "-std=c++17", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                        lib, "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


import pytest  # noqa: E402


@pytest.mark.gpu
def test_cpp_layer_runs_on_the_gpu(tmp_path):
    lib = build()
    cxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++")
    src = tmp_path / "prog.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "prog"
    subprocess.run([cxx, "-std=c++17", "-I", os.path.join(ROOT, "include"), str(src), lib, "-o", str(exe),
                    f"-Wl,-rpath,{os.path.dirname(lib)}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    n, level, v0 = r.stdout.split()
    # slots (1,2,3,0..) squared, rotated left by one, +0.5, summed over 4 slots:
    # 4 + 9 + 0 + 0 + 4 * 0.5 = 15; the product is left unrescaled (level 0)
    assert int(n) == 2048 and int(level) == 0
    assert abs(float(v0) - 15.0) < 1e-6
