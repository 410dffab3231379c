import gc
import json
import os
import torch
import operator
from constraintflow.lib.globals import device_mode
from constraintflow.lib.polyexp import PolyExpSparse
from constraintflow.lib.symexp import *
from constraintflow.gbcsr.sparse_tensor import SparseTensor
from constraintflow.lib.llist import Llist
from constraintflow.gbcsr.tensor_ops import *
class zono:
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_5 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0, type= type(0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_7 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		var_7 = any(binary(cse_var_7, cse_var_5, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_4 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_6 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		if(var_7):
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "then"})
			return cse_var_7, cse_var_6, cse_var_4, 
		else:
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "else"})
			var_6 = any(binary(cse_var_6, cse_var_5, operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			if(var_6):
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_2.json", {"taken": "then"})
				l_new_3_1 = 0.0
				u_new_3_1 = 0.0
				Z_new_3_1 = SymExpSparse(abs_elem.network,None, cse_var_5)
				return l_new_3_1, u_new_3_1, Z_new_3_1, 
			else:
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_2.json", {"taken": "else"})
				cse_var_2 = binary(cse_var_6, cse_var_7, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_3 = binary(cse_var_6, cse_var_7, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				l_new_4_2 = binary(cse_var_2, cse_var_3, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_22 = binary(cse_var_6, cse_var_4.get_const(), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_0 = cse_var_4.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_23 = binary(repeat((cse_var_6).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), symexp_0.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				var_2 = get_new_eps(abs_elem.network, torch.tensor([batch_size,curr_size,]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_20 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=1, type= type(1)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), var_2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_1 = var_2.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_21 = symexp_1.expand_symexp_mat(SymExpSparse.count)
				cse_var_17 = binary(cse_var_22, cse_var_3, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_19 = binary(cse_var_23.expand_symexp_mat(SymExpSparse.count), repeat((cse_var_3).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_1 = binary(cse_var_2, binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=2, type= type(2)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), cse_var_3, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_16 = binary(cse_var_1, cse_var_20, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_18 = binary(repeat((cse_var_1).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_21.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_2 = SymExpSparse(abs_elem.network,binary(cse_var_19.expand_symexp_mat(SymExpSparse.count), cse_var_18.expand_symexp_mat(SymExpSparse.count), operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(cse_var_17, cse_var_16, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				return l_new_4_2, cse_var_6, symexp_2, 
	
	def Affine(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_11 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_12 = curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_26 = inner_prod(cse_var_12, (cse_var_11.get_const()).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_3 = cse_var_11.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_27 = inner_prod(cse_var_12, (symexp_3.expand_symexp_mat(SymExpSparse.count)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_9 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_25 = binary(cse_var_26, cse_var_9, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_4 = SymExpSparse(abs_elem.network,cse_var_27.expand_symexp_mat(SymExpSparse.count), cse_var_25)
		cse_var_15 = symexp_4.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_8 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0, type= type(0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
		cse_var_29 = convert_to_float(binary(cse_var_15, cse_var_8, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_24 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
		cse_var_28 = unary(cse_var_15, operator.neg, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_30 = binary(binary(cse_var_24, cse_var_29, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_28, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_31 = binary(cse_var_29, cse_var_15, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		l_new = binary((unary(binary(cse_var_31, cse_var_30, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.neg, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_25, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		u_new = binary(binary((cse_var_31).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_30).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_25, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		return l_new, u_new, symexp_4, 
	
