"""crispembed-b200: CrispEmbed's NomicBERT-MoE embedding path on NVIDIA B200 (sm_100a).

The product is the shared library ``libcrispembed.so`` (C ABI in include/); this
package holds its sources (csrc/), the build script, a ctypes binding and the
synthetic-model tooling used by the tests and the benchmark.
"""
__version__ = "0.1.0"
