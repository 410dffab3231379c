class Digraph: pass
