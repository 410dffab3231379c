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
class ibp:
	def Affine(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_5 = prev.dot(curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), abs_elem.get_poly_size(), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1, mats_input = 'rhs')
		cse_var_4 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_14 = binary(cse_var_5.get_const(), cse_var_4, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_11 = PolyExpSparse(abs_elem.network, cse_var_5.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None) , cse_var_14)
		cse_var_13 = Llist(abs_elem.network, [1]*(cse_var_11.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_12 = cse_var_11.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_15 = clamp(cse_var_12, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_16 = clamp(cse_var_12, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_18 = (abs_elem.get_elem('l', cse_var_13, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_19 = (abs_elem.get_elem('u', cse_var_13, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		l_new = binary(binary(inner_prod(cse_var_16, cse_var_18, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_15, cse_var_19, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_14, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		u_new = binary(binary(inner_prod(cse_var_16, cse_var_19, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_15, cse_var_18, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_14, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		return l_new, u_new, 
	
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_9 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0, type= type(0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_10 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		rewrite_new_0 = convert_to_float(binary(cse_var_10, cse_var_9, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_17 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		l_new = binary(binary(rewrite_new_0, cse_var_10, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_17, rewrite_new_0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_9, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_8 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		rewrite_new_1 = convert_to_float(binary(cse_var_8, cse_var_9, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		u_new = binary(binary(rewrite_new_1, cse_var_8, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_17, rewrite_new_1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_9, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		return l_new, u_new, 
	
	def Sigmoid(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		l_new = unary(abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), 'sigma', layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		u_new = unary(abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), 'sigma', layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		return l_new, u_new, 
	
