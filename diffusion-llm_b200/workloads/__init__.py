"""Workloads the benchmarks and tests drive the library with: a stand-in BD3-LM backbone
(``backbone``) at the reference's model sizes, and generation loops over it
(``generation``). Not part of the drop-in boundary."""
