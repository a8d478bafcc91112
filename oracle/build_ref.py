"""Recipe: compile the reference's C++ orchestrator from its own source into oracle/_ref/.

TEST INFRASTRUCTURE ONLY. The reference module (csrc/wavefront_backend.cpp of FLB-Transformer,
a torch CppExtension per its setup.py:8-12) is compiled from the source file where it lies
under $FLB_REFERENCE_DIR (default /root/reference), with the same flags (-O3), as oracle/_ref/wavefront_backend*.so. It is
used only to generate the golden fixtures under tests/golden/ in a container that has the
reference checked out; nothing on the GPU box needs it.
"""
import os
import sys

REF = os.environ.get("FLB_REFERENCE_DIR", "/root/reference")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")


def build():
    if not os.path.isdir(REF):
        raise FileNotFoundError("reference checkout not present; nothing to build")
    os.makedirs(OUT, exist_ok=True)
    from torch.utils.cpp_extension import load
    return load(name="wavefront_backend", sources=[os.path.join(REF, "csrc", "wavefront_backend.cpp")],
                extra_cflags=["-O3"], build_directory=OUT, verbose=False)


if __name__ == "__main__":
    mod = build()
    print("built", mod.__file__, file=sys.stderr)
