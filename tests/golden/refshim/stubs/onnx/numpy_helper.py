def to_array(init): return init.array
