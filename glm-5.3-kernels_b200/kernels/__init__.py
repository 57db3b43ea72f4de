# SPDX-License-Identifier: Apache-2.0
"""B200 (sm_100a) GLM-5.3 sparse-MLA decode path.

Modules keep the reference's names so either import style works:
`from kernels.titan_mla import triton_mla_sparse_attention` with the package
root on sys.path, or `import titan_mla` with this directory on sys.path.
"""
