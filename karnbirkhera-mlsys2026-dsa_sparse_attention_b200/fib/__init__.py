"""flashinfer-bench packaging of the two operators (attention and top-k
indexer) as Solution JSON files; see pack.py and solution_kernel.py."""
