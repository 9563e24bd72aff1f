"""CPU oracle for the routed-expert MoE layer -- test infrastructure only (tests/, smoke(), bench.py's
cpu_baseline leg). The product path (prismyra_b200) never imports this package."""
