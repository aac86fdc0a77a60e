"""CPU oracle for ramvamp's routed-expert FFN path: test infrastructure only."""
