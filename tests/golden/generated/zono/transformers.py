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
	def Affine(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_8 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_9 = curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_30 = inner_prod(cse_var_9, (cse_var_8.get_const()).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_0 = cse_var_8.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_31 = inner_prod(cse_var_9, (symexp_0.expand_symexp_mat(SymExpSparse.count)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_5 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_29 = binary(cse_var_30, cse_var_5, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_1 = SymExpSparse(abs_elem.network,cse_var_31.expand_symexp_mat(SymExpSparse.count), cse_var_29)
		cse_var_1 = SparseTensor([], [], 0, torch.tensor([]), dense_const=binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), type= type(binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
		cse_var_2 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
		cse_var_26 = symexp_1.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_27 = clamp(cse_var_26, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_28 = clamp(cse_var_26, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		l_new = binary(binary((binary(cse_var_28, cse_var_1, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (binary(cse_var_27, cse_var_2, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_29, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		u_new = binary(binary((binary(cse_var_28, cse_var_2, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (binary(cse_var_27, cse_var_1, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_29, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		return l_new, u_new, symexp_1, 
	
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_21 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0, type= type(0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_47 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_48 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_16 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_23 = cse_var_16.get_const()
		symexp_2 = cse_var_16.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_24 = symexp_2.expand_symexp_mat(SymExpSparse.count)
		cse_var_42 = binary(cse_var_48, cse_var_23, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_43 = binary(repeat((cse_var_48).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_24.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		var_10 = get_new_eps(abs_elem.network, torch.tensor([batch_size,curr_size,]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_44 = binary(var_10.get_const(), SparseTensor([], [], 0, torch.tensor([]), dense_const=1, type= type(1)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_3 = var_10.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_46 = symexp_3.expand_symexp_mat(SymExpSparse.count)
		cse_var_45 = binary(cse_var_48, cse_var_47, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_40 = binary(cse_var_45, cse_var_44, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_41 = binary(repeat((cse_var_45).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_46.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_19 = binary(cse_var_48, cse_var_47, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_37 = binary(cse_var_42, cse_var_19, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_39 = binary(cse_var_43.expand_symexp_mat(SymExpSparse.count), repeat((cse_var_19).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_18 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=2, type= type(2)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), cse_var_19, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_36 = binary(cse_var_40, cse_var_18, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_38 = binary(cse_var_41.expand_symexp_mat(SymExpSparse.count), repeat((cse_var_18).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_34 = binary(cse_var_37, cse_var_36, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_35 = binary(cse_var_39.expand_symexp_mat(SymExpSparse.count), cse_var_38.expand_symexp_mat(SymExpSparse.count), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_13 = SymExpSparse(abs_elem.network,None, cse_var_21)
		cse_var_14 = binary(cse_var_48, cse_var_21, operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_32 = where(cse_var_14, cse_var_13.get_const(), cse_var_34, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_4 = cse_var_13.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_33 = where(repeat((cse_var_14).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), symexp_4.expand_symexp_mat(SymExpSparse.count), cse_var_35.expand_symexp_mat(SymExpSparse.count), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_11 = binary(cse_var_47, cse_var_21, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_5 = SymExpSparse(abs_elem.network,where(repeat((cse_var_11).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_24.expand_symexp_mat(SymExpSparse.count), cse_var_33.expand_symexp_mat(SymExpSparse.count), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), where(cse_var_11, cse_var_23, cse_var_32, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		return cse_var_21, cse_var_21, symexp_5, 
	
