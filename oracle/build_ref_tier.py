"""TEST/BASELINE INFRASTRUCTURE ONLY -- build the reference's CPU expert tier into oracle/_ref/.

Compiles kernels/cpu_avx2/ft_tier_ext.cpp (+ ft_core.h) from the reference tree, unchanged, with
torch.utils.cpp_extension.load and the flags the reference itself uses (ct/ct_vllm.py:38-39:
-O3 -std=c++17), except that -march=native is replaced by two portable ISA levels so the prebuilt
extension runs on whatever host CPU the GPU box has:
  tier_v3  -march=x86-64-v3 (AVX2/FMA/F16C: everything ft_core.h's intrinsics need)
  tier_v4  -march=x86-64-v4 (adds AVX-512; picked at run time when the host supports it)
Only a machine with the reference tree can run this; machines without it (the GPU box) use the prebuilt .so
files.

usage: python oracle/build_ref_tier.py [--ref REFERENCE_TREE] [--variants v3,v4]
(REFERENCE_TREE defaults to $DSV41_REFERENCE, else a checkout named `reference` beside this repository)
"""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    sibling = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    ap.add_argument("--ref", default=os.environ.get("DSV41_REFERENCE", sibling))
    ap.add_argument("--variants", default="v3,v4")
    a = ap.parse_args()
    src = os.path.join(a.ref, "kernels", "cpu_avx2")
    if not os.path.exists(os.path.join(src, "ft_tier_ext.cpp")):
        print(f"reference CPU tier not found under {src}; nothing built", file=sys.stderr)
        return 1
    from torch.utils.cpp_extension import load

    for v in a.variants.split(","):
        d = os.path.join(HERE, "_ref", f"tier_{v}")
        os.makedirs(d, exist_ok=True)
        load(name="ft_tier_host", sources=[os.path.join(src, "ft_tier_ext.cpp")], build_directory=d,
             extra_cflags=["-O3", f"-march=x86-64-{v}", "-std=c++17", "-I" + src],
             extra_ldflags=["-lpthread"], verbose=False)
        print("built", d)
    return 0


if __name__ == "__main__":
    sys.exit(main())
