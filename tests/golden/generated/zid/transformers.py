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
class zid:
	def Affine(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		var_26 = any(binary(curr.get_metadata('last_layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), SparseTensor([], [], 0, torch.tensor([]), dense_const=1, type= type(1)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([1, curr_size])), operator.eq, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_1 = SymExpSparse(abs_elem.network,None, SparseTensor([], [], 0, torch.tensor([]), dense_const=0, type= type(0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])))
		cse_var_13 = curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_33 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_34 = prev.dot(cse_var_13, abs_elem.get_poly_size(), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1, mats_input = 'rhs')
		cse_var_89 = binary(cse_var_34.get_const(), cse_var_33, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_110 = cse_var_34.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_75 = PolyExpSparse(abs_elem.network, cse_var_110 , cse_var_89)
		if(var_26):
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "then"})
			cse_var_177 = binary(get_dims(cse_var_110, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), 1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop1 = False
			cse_var_23 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size]))
			cse_var_181 = unary(Llist(abs_elem.network, [1]*(cse_var_177), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist()).get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.neg, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_180 = Llist(abs_elem.network, [1]*(cse_var_177), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
			cse_var_182 = abs_elem.get_elem('L', cse_var_180, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_183 = abs_elem.get_elem('U', cse_var_180, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_185 = cse_var_183.get_const()
			cse_var_184 = cse_var_183.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_187 = cse_var_182.get_const()
			cse_var_186 = cse_var_182.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			phi_trav_exp1_2_1 = cse_var_75
			while_iteration = -1
			while(True):
				while_iteration += 1
				cse_var_37 = phi_trav_exp1_2_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				vertices1_2_1 = binary(cse_var_37, cse_var_23, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices_stop_default1 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_stop_temp1 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop1, type= type(vertices_stop1)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default1, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices1_2_2 = binary(vertices1_2_1, unary(vertices_stop_temp1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				if(unary(any(vertices1_2_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
					break
				priority_vertices1 = get_max_priority(cse_var_181, vertices1_2_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_final_stop1 = binary(vertices_stop_temp1, repeat(unary(priority_vertices1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				polyexp_stop1 = filter_trav_exp_stop(phi_trav_exp1_2_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				polyexp_not_stop1 = filter_trav_exp_not_stop(phi_trav_exp1_2_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				cse_var_154 = polyexp_not_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_151 = (cse_var_154).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_146 = clamp(cse_var_154, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_148 = clamp(cse_var_154, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_142 = clamp(cse_var_151, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_144 = clamp(cse_var_151, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_102 = binary(inner_prod(cse_var_148, (cse_var_187).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_146, (cse_var_185).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_103 = binary(inner_prod((cse_var_144).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_186).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_142).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_184).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_101 = binary(cse_var_102, polyexp_not_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				trav_exp1_5_3 = PolyExpSparse(abs_elem.network, binary(cse_var_103, polyexp_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_101, polyexp_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				phi_trav_exp1_2_1 = trav_exp1_5_3
			if dummy_mode:
				json_obj = {"num_iterations": while_iteration}
				save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
			cse_var_35 = Llist(abs_elem.network, [1]*(phi_trav_exp1_2_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
			cse_var_155 = phi_trav_exp1_2_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			l_new_3_0 = binary(binary(inner_prod(clamp(cse_var_155, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_35, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_155, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_35, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp1_2_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop2 = False
			phi_trav_exp2_6_1 = cse_var_75
			while_iteration = -1
			while(True):
				while_iteration += 1
				cse_var_24 = phi_trav_exp2_6_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				vertices2_6_1 = binary(cse_var_24, cse_var_23, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices_stop_default2 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_stop_temp2 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop2, type= type(vertices_stop2)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default2, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices2_6_2 = binary(vertices2_6_1, unary(vertices_stop_temp2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				if(unary(any(vertices2_6_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
					break
				priority_vertices2 = get_max_priority(cse_var_181, vertices2_6_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_final_stop2 = binary(vertices_stop_temp2, repeat(unary(priority_vertices2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				polyexp_stop2 = filter_trav_exp_stop(phi_trav_exp2_6_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				polyexp_not_stop2 = filter_trav_exp_not_stop(phi_trav_exp2_6_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				cse_var_139 = polyexp_not_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_136 = (cse_var_139).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_131 = clamp(cse_var_139, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_133 = clamp(cse_var_139, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_127 = clamp(cse_var_136, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_129 = clamp(cse_var_136, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_93 = binary(inner_prod(cse_var_133, (cse_var_185).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_131, (cse_var_187).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_94 = binary(inner_prod((cse_var_129).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_184).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_127).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_186).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_92 = binary(cse_var_93, polyexp_not_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				trav_exp2_9_3 = PolyExpSparse(abs_elem.network, binary(cse_var_94, polyexp_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_92, polyexp_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				phi_trav_exp2_6_1 = trav_exp2_9_3
			if dummy_mode:
				json_obj = {"num_iterations": while_iteration}
				save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
			cse_var_21 = Llist(abs_elem.network, [1]*(phi_trav_exp2_6_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
			cse_var_140 = phi_trav_exp2_6_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			u_new_7_0 = binary(binary(inner_prod(clamp(cse_var_140, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_21, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_140, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_21, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp2_6_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			return l_new_3_0, u_new_7_0, cse_var_75, cse_var_75, cse_var_1, 
		else:
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "else"})
			var_25 = any(binary(curr.get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), SparseTensor([], [], 0, torch.tensor([]), dense_const=4, type= type(4)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([1, curr_size])), operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			if(var_25):
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_10.json", {"taken": "then"})
				cse_var_12 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_124 = inner_prod(cse_var_13, (cse_var_12.get_const()).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_0 = cse_var_12.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_125 = inner_prod(cse_var_13, (symexp_0.expand_symexp_mat(SymExpSparse.count)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_123 = binary(cse_var_124, cse_var_33, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_1 = SymExpSparse(abs_elem.network,cse_var_125.expand_symexp_mat(SymExpSparse.count), cse_var_123)
				cse_var_6 = SparseTensor([], [], 0, torch.tensor([]), dense_const=binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), type= type(binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
				cse_var_7 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, SymExpSparse.count]))
				cse_var_91 = symexp_1.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_121 = clamp(cse_var_91, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_122 = clamp(cse_var_91, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				l_new_11_1 = binary(binary((binary(cse_var_122, cse_var_6, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (binary(cse_var_121, cse_var_7, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_123, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				u_new_11_1 = binary(binary((binary(cse_var_122, cse_var_7, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (binary(cse_var_121, cse_var_6, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).sum(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_123, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				return l_new_11_1, u_new_11_1, cse_var_75, cse_var_75, symexp_1, 
			else:
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_10.json", {"taken": "else"})
				cse_var_88 = Llist(abs_elem.network, [1]*(cse_var_75.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
				cse_var_87 = cse_var_75.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_119 = clamp(cse_var_87, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_120 = clamp(cse_var_87, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_175 = (abs_elem.get_elem('l', cse_var_88, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_176 = (abs_elem.get_elem('u', cse_var_88, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				l_new_12_2 = binary(binary(inner_prod(cse_var_120, cse_var_175, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_119, cse_var_176, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_89, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				u_new_12_2 = binary(binary(inner_prod(cse_var_120, cse_var_176, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_119, cse_var_175, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_89, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				return l_new_12_2, u_new_12_2, cse_var_75, cse_var_75, cse_var_1, 
	
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		var_50 = any(binary(curr.get_metadata('last_layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), SparseTensor([], [], 0, torch.tensor([]), dense_const=1, type= type(1)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([1, curr_size])), operator.eq, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_72 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_44 = SymExpSparse(abs_elem.network,None, cse_var_72)
		cse_var_62 = PolyExpSparse(abs_elem.network, 0.0, cse_var_72)
		cse_var_51 = cse_var_62.get_const()
		cse_var_172 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_171 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_79 = binary(cse_var_172, cse_var_171, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_178 = binary(cse_var_172, cse_var_171, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_52 = binary(cse_var_178, cse_var_79, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_53 = cse_var_62.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_63 = binary(cse_var_172, cse_var_72, operator.lt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_54 = repeat((cse_var_63).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_86 = binary(cse_var_171, cse_var_72, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_55 = repeat((cse_var_86).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_66 = binary(cse_var_172, cse_var_79, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_56 = repeat((cse_var_66).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_68 = prev.convert_to_poly(abs_elem)
		cse_var_84 = repeat(cse_var_68.get_const(), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_85 = repeat(cse_var_68.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_67 = PolyExpSparse(abs_elem.network, 0.0, 0.0)
		cse_var_69 = binary(binary(cse_var_171, cse_var_172, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_72, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_174 = convert_to_float(cse_var_69)
		rewrite_new_0 = repeat((cse_var_174).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_173 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_179 = binary(cse_var_173, cse_var_174, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_57 = PolyExpSparse(abs_elem.network, binary(binary(rewrite_new_0, cse_var_85, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), repeat((binary(cse_var_179, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_67.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), type= type(cse_var_67.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None))).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(binary(cse_var_174, cse_var_84, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(cse_var_179, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_67.get_const(), type= type(cse_var_67.get_const())).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_117 = binary(cse_var_66, cse_var_84, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_118 = binary(cse_var_56, cse_var_85, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		rewrite_new_2 = convert_to_float(binary(cse_var_172, cse_var_72, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_82 = binary(binary(rewrite_new_2, cse_var_172, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_173, rewrite_new_2, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_72, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		rewrite_new_3 = convert_to_float(cse_var_86)
		cse_var_83 = binary(binary(rewrite_new_3, cse_var_171, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_173, rewrite_new_3, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_72, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_116 = binary(cse_var_117, cse_var_52, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_114 = where(cse_var_63, cse_var_51, cse_var_116, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_115 = where(cse_var_54, cse_var_53, cse_var_118, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_111 = PolyExpSparse(abs_elem.network, where(cse_var_55, cse_var_85, cse_var_115, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , where(cse_var_86, cse_var_84, cse_var_114, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		if(var_50):
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "then"})
			return cse_var_83, cse_var_82, cse_var_57, cse_var_111, cse_var_44, 
		else:
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "else"})
			var_49 = any(binary(curr.get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), SparseTensor([], [], 0, torch.tensor([]), dense_const=4, type= type(4)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([1, curr_size])), operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			if(var_49):
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_2.json", {"taken": "then"})
				cse_var_45 = abs_elem.get_elem('Z', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_77 = cse_var_45.get_const()
				symexp_2 = cse_var_45.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_78 = symexp_2.expand_symexp_mat(SymExpSparse.count)
				cse_var_166 = binary(cse_var_172, cse_var_77, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_167 = binary(repeat((cse_var_172).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_78.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				var_40 = get_new_eps(abs_elem.network, torch.tensor([batch_size,curr_size,]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_168 = binary(var_40.get_const(), cse_var_173, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_3 = var_40.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_170 = symexp_3.expand_symexp_mat(SymExpSparse.count)
				cse_var_164 = binary(cse_var_178, cse_var_168, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_165 = binary(repeat((cse_var_178).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_170.expand_symexp_mat(SymExpSparse.count), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_161 = binary(cse_var_166, cse_var_79, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_163 = binary(cse_var_167.expand_symexp_mat(SymExpSparse.count), repeat((cse_var_79).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_46 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=2, type= type(2)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), cse_var_79, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_160 = binary(cse_var_164, cse_var_46, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_162 = binary(cse_var_165.expand_symexp_mat(SymExpSparse.count), repeat((cse_var_46).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_158 = binary(cse_var_161, cse_var_160, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_159 = binary(cse_var_163.expand_symexp_mat(SymExpSparse.count), cse_var_162.expand_symexp_mat(SymExpSparse.count), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_43 = binary(cse_var_172, cse_var_72, operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_156 = where(cse_var_43, cse_var_44.get_const(), cse_var_158, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_4 = cse_var_44.get_mat(SymExpSparse.count, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_157 = where(repeat((cse_var_43).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), symexp_4.expand_symexp_mat(SymExpSparse.count), cse_var_159.expand_symexp_mat(SymExpSparse.count), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_41 = binary(cse_var_171, cse_var_72, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				symexp_5 = SymExpSparse(abs_elem.network,where(repeat((cse_var_41).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, SymExpSparse.count]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_78.expand_symexp_mat(SymExpSparse.count), cse_var_157.expand_symexp_mat(SymExpSparse.count), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), where(cse_var_41, cse_var_77, cse_var_156, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				return cse_var_83, cse_var_82, cse_var_57, cse_var_111, symexp_5, 
			else:
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_2.json", {"taken": "else"})
				return cse_var_83, cse_var_82, cse_var_57, cse_var_111, cse_var_44, 
	
