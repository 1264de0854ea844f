"""CPU oracle for the taccel golden simulator: TEST INFRASTRUCTURE ONLY.

A NumPy restatement of the reference's per-instruction execute loop
(SayatAbdikul/LLM_accelerator, software/taccel/golden_model), pinned to the
reference by the golden vectors in tests/golden.  Only tests/,
__graft_entry__.smoke() and the CPU-baseline legs of bench.py may import it;
the engine in llm_accelerator_b200 never does.
"""
