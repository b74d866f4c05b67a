"""Drop-in kernel wrappers with the reference's names and signatures
(``kbench/core/kernels/*.py`` of the reference project), backed by the sm_100a C ABI."""
