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
class polyzono:
	def Affine(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_31 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_32 = curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_127 = inner_prod(cse_var_32, (cse_var_31.get_const()).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_0 = cse_var_31.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_128 = inner_prod(cse_var_32, (symexp_0.expand_symexp_mat(SymExpSparse.count)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_30 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_126 = binary(cse_var_127, cse_var_30, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_1 = SymExpSparse(abs_elem.network,cse_var_128.expand_symexp_mat(SymExpSparse.count), cse_var_126)
		cse_var_24 = prev.dot(cse_var_32, abs_elem.get_poly_size(), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1, mats_input = 'rhs')
		cse_var_88 = cse_var_24.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_58 = PolyExpSparse(abs_elem.network, cse_var_88 , binary(cse_var_24.get_const(), cse_var_30, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_148 = binary(get_dims(cse_var_88, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), 1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		vertices_stop1 = False
		cse_var_14 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size]))
		cse_var_152 = unary(Llist(abs_elem.network, [1]*(cse_var_148), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist()).get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.neg, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_151 = Llist(abs_elem.network, [1]*(cse_var_148), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_153 = abs_elem.get_elem('L', cse_var_151, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_154 = abs_elem.get_elem('U', cse_var_151, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_156 = cse_var_154.get_const()
		cse_var_155 = cse_var_154.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_158 = cse_var_153.get_const()
		cse_var_157 = cse_var_153.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		phi_trav_exp1_1_1 = cse_var_58
		while_iteration = -1
		while(True):
			while_iteration += 1
			cse_var_29 = phi_trav_exp1_1_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			vertices1_1_1 = binary(cse_var_29, cse_var_14, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop_default1 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_stop_temp1 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop1, type= type(vertices_stop1)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default1, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices1_1_2 = binary(vertices1_1_1, unary(vertices_stop_temp1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			if(unary(any(vertices1_1_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
				break
			priority_vertices1 = get_max_priority(cse_var_152, vertices1_1_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_final_stop1 = binary(vertices_stop_temp1, repeat(unary(priority_vertices1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			polyexp_stop1 = filter_trav_exp_stop(phi_trav_exp1_1_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			polyexp_not_stop1 = filter_trav_exp_not_stop(phi_trav_exp1_1_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_124 = polyexp_not_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_121 = (cse_var_124).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_116 = clamp(cse_var_124, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_118 = clamp(cse_var_124, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_112 = clamp(cse_var_121, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_114 = clamp(cse_var_121, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_80 = binary(inner_prod(cse_var_118, (cse_var_158).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_116, (cse_var_156).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_81 = binary(inner_prod((cse_var_114).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_157).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_112).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_155).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_79 = binary(cse_var_80, polyexp_not_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			trav_exp1_4_3 = PolyExpSparse(abs_elem.network, binary(cse_var_81, polyexp_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_79, polyexp_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
			phi_trav_exp1_1_1 = trav_exp1_4_3
		if dummy_mode:
			json_obj = {"num_iterations": while_iteration}
			save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
		cse_var_10 = SparseTensor([], [], 0, torch.tensor([]), dense_const=binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), type= type(binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
		cse_var_11 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
		cse_var_26 = Llist(abs_elem.network, [1]*(phi_trav_exp1_1_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_125 = phi_trav_exp1_1_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_78 = symexp_1.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_109 = clamp(cse_var_78, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_110 = clamp(cse_var_78, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		l_new = cf_max(binary(binary((binary(cse_var_110, cse_var_10, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (binary(cse_var_109, cse_var_11, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_126, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(inner_prod(clamp(cse_var_125, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_26, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_125, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_26, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp1_1_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		vertices_stop2 = False
		phi_trav_exp2_5_1 = cse_var_58
		while_iteration = -1
		while(True):
			while_iteration += 1
			cse_var_15 = phi_trav_exp2_5_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			vertices2_5_1 = binary(cse_var_15, cse_var_14, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop_default2 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_stop_temp2 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop2, type= type(vertices_stop2)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default2, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices2_5_2 = binary(vertices2_5_1, unary(vertices_stop_temp2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			if(unary(any(vertices2_5_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
				break
			priority_vertices2 = get_max_priority(cse_var_152, vertices2_5_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_final_stop2 = binary(vertices_stop_temp2, repeat(unary(priority_vertices2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			polyexp_stop2 = filter_trav_exp_stop(phi_trav_exp2_5_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			polyexp_not_stop2 = filter_trav_exp_not_stop(phi_trav_exp2_5_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_107 = polyexp_not_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_104 = (cse_var_107).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_99 = clamp(cse_var_107, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_101 = clamp(cse_var_107, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_95 = clamp(cse_var_104, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_97 = clamp(cse_var_104, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_69 = binary(inner_prod(cse_var_101, (cse_var_156).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_99, (cse_var_158).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_70 = binary(inner_prod((cse_var_97).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_155).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_95).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_157).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_68 = binary(cse_var_69, polyexp_not_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			trav_exp2_8_3 = PolyExpSparse(abs_elem.network, binary(cse_var_70, polyexp_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_68, polyexp_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
			phi_trav_exp2_5_1 = trav_exp2_8_3
		if dummy_mode:
			json_obj = {"num_iterations": while_iteration}
			save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
		cse_var_8 = Llist(abs_elem.network, [1]*(phi_trav_exp2_5_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_108 = phi_trav_exp2_5_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		u_new = cf_min(binary(binary((binary(cse_var_110, cse_var_11, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (binary(cse_var_109, cse_var_10, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_126, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(inner_prod(clamp(cse_var_108, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_8, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_108, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_8, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp2_5_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		return l_new, u_new, cse_var_58, cse_var_58, symexp_1, 
	
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_144 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_56 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_65 = binary(cse_var_144, cse_var_56, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		rewrite_new_0 = convert_to_float(cse_var_65)
		cse_var_147 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		l_new = binary(binary(rewrite_new_0, cse_var_144, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_147, rewrite_new_0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_56, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_145 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		rewrite_new_1 = convert_to_float(binary(cse_var_145, cse_var_56, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		u_new = binary(binary(rewrite_new_1, cse_var_145, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_147, rewrite_new_1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_56, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_52 = prev.convert_to_poly(abs_elem)
		cse_var_66 = repeat(cse_var_52.get_const(), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_67 = repeat(cse_var_52.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_51 = PolyExpSparse(abs_elem.network, 0.0, 0.0)
		cse_var_53 = binary(binary(cse_var_144, cse_var_145, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_56, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_146 = convert_to_float(cse_var_53)
		rewrite_new_2 = repeat((cse_var_146).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_150 = binary(cse_var_147, cse_var_146, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		L_new = PolyExpSparse(abs_elem.network, binary(binary(rewrite_new_2, cse_var_67, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), repeat((binary(cse_var_150, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_51.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), type= type(cse_var_51.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None))).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(binary(cse_var_146, cse_var_66, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(cse_var_150, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_51.get_const(), type= type(cse_var_51.get_const())).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_63 = binary(cse_var_145, cse_var_144, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_50 = binary(cse_var_145, cse_var_63, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_92 = binary(cse_var_50, cse_var_66, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_93 = binary(repeat((cse_var_50).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_67, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_149 = binary(cse_var_145, cse_var_144, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_91 = binary(cse_var_92, binary(cse_var_149, cse_var_63, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_46 = PolyExpSparse(abs_elem.network, 0.0, cse_var_56)
		cse_var_47 = binary(cse_var_145, cse_var_56, operator.lt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_89 = where(cse_var_47, cse_var_46.get_const(), cse_var_91, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_90 = where(repeat((cse_var_47).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_46.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), cse_var_93, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		U_new = PolyExpSparse(abs_elem.network, where(repeat((cse_var_65).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_67, cse_var_90, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , where(cse_var_65, cse_var_66, cse_var_89, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_38 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_61 = cse_var_38.get_const()
		symexp_2 = cse_var_38.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_62 = symexp_2.expand_symexp_mat(SymExpSparse.count)
		cse_var_139 = binary(cse_var_145, cse_var_61, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_140 = binary(repeat((cse_var_145).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_62.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		var_26 = get_new_eps(abs_elem.network, torch.tensor([batch_size,curr_size,]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_141 = binary(var_26.get_const(), cse_var_147, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_3 = var_26.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_143 = symexp_3.expand_symexp_mat(SymExpSparse.count)
		cse_var_137 = binary(cse_var_149, cse_var_141, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_138 = binary(repeat((cse_var_149).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_143.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_134 = binary(cse_var_139, cse_var_63, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_136 = binary(cse_var_140.expand_symexp_mat(SymExpSparse.count), repeat((cse_var_63).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_39 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=2, type= type(2)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), cse_var_63, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_133 = binary(cse_var_137, cse_var_39, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_135 = binary(cse_var_138.expand_symexp_mat(SymExpSparse.count), repeat((cse_var_39).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_131 = binary(cse_var_134, cse_var_133, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_132 = binary(cse_var_136.expand_symexp_mat(SymExpSparse.count), cse_var_135.expand_symexp_mat(SymExpSparse.count), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_36 = SymExpSparse(abs_elem.network,None, cse_var_56)
		cse_var_37 = binary(cse_var_145, cse_var_56, operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_129 = where(cse_var_37, cse_var_36.get_const(), cse_var_131, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_4 = cse_var_36.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_130 = where(repeat((cse_var_37).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), symexp_4.expand_symexp_mat(SymExpSparse.count), cse_var_132.expand_symexp_mat(SymExpSparse.count), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_34 = binary(cse_var_144, cse_var_56, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		symexp_5 = SymExpSparse(abs_elem.network,where(repeat((cse_var_34).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_62.expand_symexp_mat(SymExpSparse.count), cse_var_130.expand_symexp_mat(SymExpSparse.count), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), where(cse_var_34, cse_var_61, cse_var_129, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		return l_new, u_new, L_new, U_new, symexp_5, 
	
